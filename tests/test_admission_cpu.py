"""KV admission control: requests are admitted against their own worst-case block count.

A pool smaller than max_num_seqs full-length requests must not run dry in the
middle of a generation: the scheduler admits a waiting request only when the
blocks not promised to running requests cover the new one's prompt, all of its
output and the verify look-ahead; the others wait for running ones to finish.
"""
import numpy as np
import pytest

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine


def _engine(num_blocks, method="hybrid"):
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    cfg = EngineConfig(model=m, spec=SpecConfig(method=method, k=4), device="cpu", cuda_graphs=False,
                       cache=CacheConfig(max_model_len=256, block_size=16, num_blocks=num_blocks), max_num_seqs=4)
    return LLMEngine(cfg)


def test_small_pool_serialises_requests_and_matches_a_large_pool():
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 512, int(rng.integers(40, 90))) for _ in range(5)]
    want = _engine(0, "none").generate(prompts, max_new_tokens=40)
    small = _engine(20, "none")  # about two of these requests at a time, not four
    running = []
    orig = small.step

    def spy():
        st = orig()
        running.append(len(small.running))
        used = small.pool.num_blocks - 1 - small.pool.free
        assert used <= small.pool.num_blocks - 1
        return st

    small.step = spy
    got = small.generate(prompts, max_new_tokens=40)
    assert got == want
    assert max(running) < 4  # the pool, not max_num_seqs, bounded the concurrency


def test_reservation_covers_the_verify_look_ahead():
    eng = _engine(0)
    rid = eng.add_request(np.arange(50) % 512, max_new_tokens=30)
    r = eng.waiting[0]
    # the decode step keeps blocks for committed + 2k + 2 positions; committed reaches prompt + output
    assert eng._reservation(r) * eng.block_size >= 50 + 30 + 2 * eng.k + 2
    assert rid == r.rid


def test_request_larger_than_the_pool_is_refused_not_deadlocked():
    eng = _engine(6, "none")
    eng.add_request(np.arange(200) % 512, max_new_tokens=40)
    with pytest.raises(MemoryError):
        eng.step()


def test_rope_table_covers_max_model_len():
    """A 128k prompt plus its output runs past a 131072-entry RoPE table: the engine extends the table to
    every position a max_model_len request can write (the Kimi-K2 benchmark layout)."""
    m = shrink(llama3_8b_config(), layers=1, hidden=64, vocab=256)
    m.dtype = "float32"
    m.max_position = 300
    cfg = EngineConfig(model=m, spec=SpecConfig(method="none", k=0), device="cpu", cuda_graphs=False,
                       cache=CacheConfig(max_model_len=512, block_size=16), max_num_seqs=2)
    eng = LLMEngine(cfg)
    assert eng.model.cos_sin.shape[0] >= 512 + 2
    out = eng.generate([np.arange(400) % 256], max_new_tokens=100)  # positions 400..499 exist in the table
    assert len(out[0]) == 100
