"""Chunked prefill on the GPU kernels: prompt chunks attend over the cached part of their prompt (paged
attention, MLA + DSA indexer) and the engine generates what a whole-prompt prefill generates; a
recurrent-state model prefills the long prompt whole."""
import numpy as np
import pytest

from vllm_suffix_hybrid_b200.engine.config import (CacheConfig, EngineConfig, SpecConfig, deepseek_v32_config,
                                                   llama3_8b_config, qwen3_next_config, shrink)
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", ["llama", "deepseek_v32", "qwen3_next"])
def test_chunked_prefill_matches_whole_prompt_prefill(name):
    base = {"llama": llama3_8b_config, "deepseek_v32": deepseek_v32_config, "qwen3_next": qwen3_next_config}[name]()
    m = shrink(base, layers=3, hidden=256, vocab=1024)
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 1024, int(n)) for n in (60, 700, 90)]
    outs, kinds = [], []
    for chunked in (False, True):
        cfg = EngineConfig(model=m, spec=SpecConfig(method="hybrid", k=3), cache=CacheConfig(max_model_len=1024),
                           max_num_seqs=4, device="cuda", cuda_graphs=True, max_prefill_tokens=256,
                           chunked_prefill=chunked)
        eng = LLMEngine(cfg)
        outs.append(eng.generate(prompts, max_new_tokens=16))
        kinds.append(sum(s.kind == "prefill" for s in eng.stats))
    assert all(len(o) == 16 for o in outs[1])
    agree = np.mean([a == b for a, b in zip(outs[0], outs[1])])
    assert agree >= 2 / 3, (outs[0], outs[1])  # a different summation order may flip a bf16 near-tie
    if name == "qwen3_next":
        assert kinds[0] == kinds[1]  # recurrent state: the long prompt is prefilled whole
    else:
        assert kinds[1] > kinds[0]  # the 700-token prompt took three 256-token chunks
