"""NVFP4-screened LM head: the screen + exact re-score picks the same greedy token as the bf16 head
whenever the true argmax is among the screened candidates, and the engine decodes identically."""
import numpy as np
import torch

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
from vllm_suffix_hybrid_b200.models.lm_head import ScreenedHead


def test_rescore_recovers_exact_argmax():
    torch.manual_seed(0)
    V, H, M = 1000, 256, 12
    w = (torch.randn(V, H) * 0.05).to(torch.bfloat16)
    x = torch.randn(M, H).to(torch.bfloat16)
    head = ScreenedHead(w)
    val, ids = head.best(x)
    exact = (x.float() @ w.float().t()).bfloat16().float()
    assert torch.equal(ids, exact.argmax(-1))  # first occurrence among bf16 ties, like the bf16 head
    assert torch.equal(val, exact.max(-1).values)


def test_engine_with_screened_head_matches_bf16_head(monkeypatch):
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "bfloat16"
    cfg = lambda: EngineConfig(model=m, spec=SpecConfig(method="none"), cache=CacheConfig(max_model_len=128),
                               max_num_seqs=2, device="cpu", cuda_graphs=False)
    rng = np.random.default_rng(2)
    prompts = [rng.integers(0, 512, 12) for _ in range(2)]
    base = LLMEngine(cfg()).generate(prompts, max_new_tokens=8)
    monkeypatch.setenv("SUFFIX_NVFP4_LMHEAD", "1")
    eng = LLMEngine(cfg())
    assert getattr(eng.model, "lm_screen", None) is not None
    got = eng.generate(prompts, max_new_tokens=8)
    assert got == base
