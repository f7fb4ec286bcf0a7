"""Engine on a B200: speculative decoding (eager and CUDA-graph) reproduces plain greedy decoding.

Runs in batch-invariant mode: bit-exact agreement between a k+1-token verify
window and one-token decoding needs kernels whose per-row reduction order
does not depend on the number of rows in the call.
"""
import os

import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _batch_invariant(monkeypatch):
    monkeypatch.setenv("SH_BATCH_INVARIANT", "1")


def run(method, graphs, prompts, k=5, new=24):
    cfg = EngineConfig(model=shrink(llama3_8b_config(), layers=2, hidden=512, vocab=4096),
                       spec=SpecConfig(method=method, k=k), cache=CacheConfig(max_model_len=1024),
                       max_num_seqs=4, device="cuda", cuda_graphs=graphs)
    eng = LLMEngine(cfg)
    return eng.generate(prompts, max_new_tokens=new), eng


def test_spec_modes_match_greedy():
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 4096, int(n)) for n in (100, 70, 130, 64, 33)]
    base, _ = run("none", False, prompts)
    for method in ("hybrid", "native", "suffix", "ngram"):
        for graphs in (False, True):
            got, eng = run(method, graphs, prompts)
            agree = np.mean([a == b for a, b in zip(got, base)])
            assert agree == 1.0, (method, graphs, got, base)


@pytest.mark.parametrize("graphs", [False, True])
def test_qwen3_next_oracle_drafts_on_gpu(graphs):
    from vllm_suffix_hybrid_b200.engine.config import qwen3_next_config

    m = shrink(qwen3_next_config(), layers=4, hidden=256, vocab=1024)
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, 1024, int(n)) for n in (40, 23, 64)]
    base_cfg = EngineConfig(model=m, spec=SpecConfig(method="none"), cache=CacheConfig(max_model_len=512),
                            max_num_seqs=4, device="cuda", cuda_graphs=False)
    base = LLMEngine(base_cfg).generate(prompts, max_new_tokens=16)
    truth = {f"req-{i}": b for i, b in enumerate(base)}
    cfg = EngineConfig(model=m, spec=SpecConfig(method="external", k=4), cache=CacheConfig(max_model_len=512),
                       max_num_seqs=4, device="cuda", cuda_graphs=graphs)
    eng = LLMEngine(cfg)
    r = np.random.default_rng(5)

    def oracle(reqs):
        out = []
        for q in reqs:
            cont = list(truth[q.rid][len(q.output):len(q.output) + 4]) + [0] * 4
            cont = cont[:4]
            bad = int(r.integers(0, 6))
            if bad < 4:
                cont[bad] = (cont[bad] + 1) % 1024
            out.append(cont)
        return out

    eng.external_proposer = oracle
    got = eng.generate(prompts, max_new_tokens=16)
    agree = np.mean([a == b for a, b in zip(got, base)])
    assert agree == 1.0, (got, base)
    assert eng.spec_stats()["mean_accept_len"] > 1.5


@pytest.mark.parametrize("method", ["suffix", "hybrid"])
@pytest.mark.parametrize("graphs", [False, True])
def test_async_scheduling_matches_greedy_on_gpu(method, graphs):
    """Lag-1 drafting with the device-side resolve (spec_advance kernel) inside the pipelined step."""
    rng = np.random.default_rng(1)
    prompts = [rng.integers(0, 4096, int(n)) for n in (100, 70, 130, 64, 33)]
    base, _ = run("none", False, prompts, new=32)
    m = shrink(llama3_8b_config(), layers=2, hidden=512, vocab=4096)
    cfg = EngineConfig(model=m, spec=SpecConfig(method=method, k=5, async_scheduling=True),
                       cache=CacheConfig(max_model_len=1024), max_num_seqs=4, device="cuda", cuda_graphs=graphs)
    eng = LLMEngine(cfg)
    eng.warm_start([np.concatenate([p, b]) for p, b in zip(prompts, base)])
    got = eng.generate(prompts, max_new_tokens=32)
    assert got == base
    assert eng.spec_stats()["mean_accept_len"] > 1.5
