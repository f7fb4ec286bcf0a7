"""Chunked prefill: a prompt longer than max_prefill_tokens is prefilled in chunks that alternate with the
running requests' decode steps, and generates what a whole-prompt prefill generates."""
import numpy as np
import pytest

from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, SpecConfig, deepseek_v32_config,
                                                   llama3_8b_config, shrink)
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine


def _cfg(model, method, chunked, budget=48):
    return EngineConfig(model=model, spec=SpecConfig(method=method, k=3), cache=CacheConfig(max_model_len=512),
                        max_num_seqs=4, device="cpu", cuda_graphs=False, max_prefill_tokens=budget,
                        chunked_prefill=chunked)


@pytest.mark.parametrize("name,method", [("llama", "none"), ("llama", "hybrid"), ("deepseek", "none")])
def test_chunked_prefill_generates_the_same_tokens(name, method):
    m = (shrink(llama3_8b_config(), layers=2, hidden=128, vocab=256) if name == "llama"
         else shrink(deepseek_v32_config(), layers=2, hidden=128, vocab=256))
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 256, n) for n in (30, 170, 20)]
    outs = []
    for chunked in (False, True):
        outs.append(LLMEngine(_cfg(m, method, chunked)).generate(prompts, max_new_tokens=10))
    assert outs[0] == outs[1]


def test_chunks_alternate_with_decode_steps():
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=256)
    eng = LLMEngine(_cfg(m, "none", True, budget=40))
    free0 = eng.pool.free
    rng = np.random.default_rng(5)
    a = eng.add_request(rng.integers(0, 256, 20), max_new_tokens=30)
    eng.step()  # short prompt: a whole-prompt prefill
    b = eng.add_request(rng.integers(0, 256, 200), max_new_tokens=5)  # 5 chunks of 40
    kinds = []
    while eng.prefilling is not None or any(r.rid == b for r in eng.waiting):
        kinds.append(eng.step().kind)
        assert len(kinds) < 30
    assert kinds.count("prefill") == 5
    # every chunk after the first follows a decode step of the running request
    assert all(kinds[i - 1] == "decode" for i, k in enumerate(kinds) if k == "prefill" and i > 0)
    _, done_a, _ = eng.poll(a)
    new_b, _, _ = eng.poll(b)
    assert len(new_b) == 1 and not done_a
    while eng.has_work():
        eng.step()
    assert len(eng.finished[b].output) == 5 and len(eng.finished[a].output) == 30
    assert eng.pool.free == free0


def test_abort_during_chunked_prefill_frees_its_blocks():
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=256)
    eng = LLMEngine(_cfg(m, "none", True, budget=40))
    free0 = eng.pool.free
    rid = eng.add_request(np.arange(150) % 256, max_new_tokens=5)
    eng.step()
    assert eng.prefilling is not None and eng.prefilling.rid == rid
    assert eng.abort_request(rid)
    assert eng.prefilling is None and eng.pool.free == free0
    assert eng.poll(rid)[1:] == (True, "abort")
    assert not eng.has_work()


def test_recurrent_models_prefill_whole_and_data_parallel_is_excluded():
    from vllm_suffix_hybrid_b200.engine.config import qwen3_next_config

    m = shrink(qwen3_next_config(), layers=2, hidden=128, vocab=256)
    eng = LLMEngine(_cfg(m, "none", True, budget=32))
    rid = eng.add_request(np.arange(100) % 256, max_new_tokens=4)
    assert not eng._chunkable(eng.waiting[0])  # GDN states prefill from the empty state only
    st = eng.step()
    assert st.kind == "prefill" and eng.prefilling is None and eng.running[0].rid == rid
    with pytest.raises(ValueError, match="attention-only"):
        eng.runner.prefill([np.arange(8)], [eng.running[0].blocks], [eng.running[0].slot], starts=[4])
