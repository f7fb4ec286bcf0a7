"""Speculative decoding with accepted drafts reproduces plain greedy decoding.

An oracle drafter proposes the true continuation (from a plain-decode run)
with a corrupted token at a random slot, so accepted lengths vary from 0 to k
and the commit paths (paged KV for attention, deferred record replay for
Gated DeltaNet state) are exercised with real acceptances.
"""
import numpy as np
import pytest

from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, SpecConfig, deepseek_v32_config,
                                                   kimi_k2_config, llama3_8b_config, qwen3_next_config, shrink)
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine


def _model(name):
    if name == "llama":
        m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    elif name == "qwen3_next":
        m = shrink(qwen3_next_config(), layers=4, hidden=128, vocab=512)
    elif name == "deepseek_v32":
        m = shrink(deepseek_v32_config(), layers=3, hidden=128, vocab=512)
    else:
        m = shrink(kimi_k2_config(), layers=3, hidden=128, vocab=512)
    m.dtype = "float32"
    m.weight_format = "bf16"
    return m


@pytest.mark.parametrize("name", ["llama", "qwen3_next", "deepseek_v32", "kimi_k2"])
def test_oracle_drafts_match_plain_decode(name, monkeypatch):
    # Batch-invariant mode: a verify window computes its rows in larger matmuls than plain decode, and the
    # DeepSeek indexer quantises its queries to e4m3, so a last-bit difference in a query can move a code and
    # change the selected keys.  Invariant mode makes every row independent of the batch.
    monkeypatch.setenv("SH_BATCH_INVARIANT", "1")
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 512, int(rng.integers(8, 30))) for _ in range(3)]
    base_cfg = EngineConfig(model=_model(name), spec=SpecConfig(method="none"), cache=CacheConfig(max_model_len=256),
                            max_num_seqs=2, device="cpu", cuda_graphs=False)
    base = LLMEngine(base_cfg).generate(prompts, max_new_tokens=24)
    truth = {f"req-{i}": b for i, b in enumerate(base)}
    k = 4
    cfg = EngineConfig(model=_model(name), spec=SpecConfig(method="external", k=k),
                       cache=CacheConfig(max_model_len=256), max_num_seqs=2, device="cpu", cuda_graphs=False)
    eng = LLMEngine(cfg)
    r = np.random.default_rng(11)

    def oracle(reqs):
        out = []
        for q in reqs:
            done = len(q.output)
            cont = list(truth[q.rid][done:done + k])
            cont += [0] * (k - len(cont))
            bad = int(r.integers(0, k + 2))  # >= k: no corruption (full accept)
            if bad < k:
                cont[bad] = (cont[bad] + 1) % 512
            out.append(cont)
        return out

    eng.external_proposer = oracle
    got = eng.generate(prompts, max_new_tokens=24)
    assert got == base
    assert eng.spec_stats()["mean_accept_len"] > 1.5
