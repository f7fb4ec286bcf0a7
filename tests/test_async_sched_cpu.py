"""Async scheduling (lag-1 drafting, SUFFIX_HYBRID_ASYNC=1) reproduces plain greedy decoding.

The suffix corpus is warm-started with the true continuations, so the lag-1 candidates are mostly right
and the device-side resolve (spec_advance) both accepts and rejects drafts.  Three prompts on two rows
make the pipeline drain and restart around a prefill and around finishing rows.
"""
import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, llama3_8b_config, shrink
from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
from vllm_suffix_hybrid_b200.ops import reference as ref


def _cfg(method, async_sched=False, graphs=False):
    m = shrink(llama3_8b_config(), layers=2, hidden=128, vocab=512)
    m.dtype = "float32"
    return EngineConfig(model=m, spec=SpecConfig(method=method, k=4, async_scheduling=async_sched),
                        cache=CacheConfig(max_model_len=256), max_num_seqs=2, device="cpu", cuda_graphs=graphs)


@pytest.mark.parametrize("method", ["suffix", "hybrid"])
def test_async_scheduling_matches_greedy(method):
    rng = np.random.default_rng(7)
    prompts = [rng.integers(0, 512, int(rng.integers(10, 30))) for _ in range(3)]
    base = LLMEngine(_cfg("none")).generate(prompts, max_new_tokens=30)
    eng = LLMEngine(_cfg(method, async_sched=True))
    assert eng._async
    eng.warm_start([np.concatenate([p, b]) for p, b in zip(prompts, base)])
    got = eng.generate(prompts, max_new_tokens=30)
    assert got == base
    st = eng.spec_stats()
    assert st["mean_accept_len"] > 1.5, st
    kinds = {s.kind for s in eng.stats}
    assert "launch" in kinds and "decode" in kinds


def test_async_ignored_for_unsupported_methods():
    eng = LLMEngine(_cfg("ngram", async_sched=True))
    assert not eng._async


def test_spec_advance_reference_cases():
    k, L = 3, 7
    out = torch.tensor([[5, 6, 9, -1], [1, -1, -1, -1], [4, 4, 4, 4]])
    acc = torch.tensor([2, 0, 3], dtype=torch.int32)
    nxt = torch.tensor([9, 1, 4])
    seq_new = torch.tensor([13, 21, 34])
    cand = torch.tensor([[5, 6, 9, 10, 11, 12, 13], [2, 3, 4, 5, 6, 7, 8], [4, 4, 4, 4, 7, 0, 0]])
    clen = torch.tensor([7, 7, 5], dtype=torch.int32)
    win, seq, real = ref.spec_advance(out, acc, nxt, seq_new, cand, clen, None, 0)
    assert win[0].tolist() == [9, 10, 11, 12] and int(real[0]) == 3  # aligned: C[3:6]
    assert win[1].tolist() == [1, -1, -1, -1] and int(real[1]) == 0  # C[0] != accepted token
    assert win[2].tolist() == [4, 7, -1, -1] and int(real[2]) == 1  # aligned, candidate runs out
    assert seq.tolist() == [13, 21, 34]
    nat = torch.tensor([[70, 71, 72], [80, 81, 82], [90, 91, 92]])
    win, _, real = ref.spec_advance(out, acc, nxt, seq_new, cand, clen, nat, 2)
    assert win[0].tolist() == [9, 10, 11, 12]  # 3 real >= 2: suffix drafts
    assert win[1].tolist() == [1, 80, 81, 82] and win[2].tolist() == [4, 90, 91, 92]  # native fallback
    # the ops wrapper (CPU path) resets bucket-padding rows
    w2 = torch.zeros(4, k + 1, dtype=torch.long)
    s2 = torch.zeros(4, dtype=torch.long)
    r2 = torch.zeros(4, dtype=torch.int32)
    pad = lambda t, v=0: torch.cat([t, torch.full((1,) + tuple(t.shape[1:]), v, dtype=t.dtype)])
    ops.spec_advance(pad(out), pad(acc), pad(nxt), pad(seq_new, 99), pad(cand), pad(clen), None, w2, s2, r2, 0, 3)
    assert w2[:3].tolist() == ref.spec_advance(out, acc, nxt, seq_new, cand, clen, None, 0)[0].tolist()
    assert w2[3].tolist() == [0, 0, 0, 0] and int(s2[3]) == 0
