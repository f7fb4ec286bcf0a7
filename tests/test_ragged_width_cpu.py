"""Adaptive verify width: a step verifies only as many tokens per row as the longest real draft.

Suffix-only drafting in ragged mode (uniform_k off) publishes each row's true
draft length, often 0 while the corpus has no match; the runner then runs the
step at width 1 + max(real drafts) instead of k + 1.  Outputs must equal the
fixed-width engine and plain greedy decoding token for token.
"""
import numpy as np

from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine


def _cfg(method, adaptive=True, k=4):
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    spec = SpecConfig(method=method, k=k, uniform_k=False, adaptive_width=adaptive)
    return EngineConfig(model=m, spec=spec, cache=CacheConfig(max_model_len=256), max_num_seqs=3, device="cpu",
                        cuda_graphs=False)


def _widths(eng, fn):
    seen = []
    orig = eng.runner.decode

    def spy(*a, **kw):
        seen.append(kw.get("width"))
        return orig(*a, **kw)

    eng.runner.decode = spy
    out = fn()
    eng.runner.decode = orig
    return out, seen


def test_adaptive_width_matches_fixed_width_and_greedy():
    rng = np.random.default_rng(11)
    prompts = [rng.integers(0, 512, int(rng.integers(12, 40))) for _ in range(4)]
    base = LLMEngine(_cfg("none")).generate(prompts, max_new_tokens=24)
    # Warm only part of the corpus: some rows get drafts, others miss (width-0 rows).
    warm = [np.concatenate([p, b]) for p, b in zip(prompts[:2], base[:2])]
    fixed = LLMEngine(_cfg("suffix", adaptive=False))
    fixed.warm_start(warm)
    want, w_fixed = _widths(fixed, lambda: fixed.generate(prompts, max_new_tokens=24))
    ragged = LLMEngine(_cfg("suffix", adaptive=True))
    ragged.warm_start(warm)
    got, w_ragged = _widths(ragged, lambda: ragged.generate(prompts, max_new_tokens=24))
    assert want == base and got == base
    assert set(w_fixed) == {5}
    assert min(w_ragged) < 5  # some steps ran narrower than k + 1
    assert 1 in w_ragged or min(w_ragged) <= 2
    assert ragged.spec_stats()["mean_accept_len"] > 1.0


def test_no_drafts_is_a_plain_decode_step():
    rng = np.random.default_rng(3)
    prompts = [rng.integers(0, 512, 20) for _ in range(2)]
    base = LLMEngine(_cfg("none")).generate(prompts, max_new_tokens=10)
    eng = LLMEngine(_cfg("suffix", adaptive=True))  # cold corpus: no drafts anywhere
    got, widths = _widths(eng, lambda: eng.generate(prompts, max_new_tokens=10))
    assert got == base
    assert widths and all(w == 1 for w in widths)
