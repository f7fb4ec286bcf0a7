"""Engine on a B200: speculative decoding (eager and CUDA-graph) reproduces plain greedy decoding."""
import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

pytestmark = pytest.mark.gpu


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
