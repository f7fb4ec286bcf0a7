"""Greedy verification oracle vs a plain PyTorch restatement of greedy rejection."""
import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200._native import rejection_greedy_accept

K = 8


def torch_greedy(draft, logits, cu, k):
    argmax = logits.float().argmax(-1)
    B = cu.shape[0]
    out = torch.full((B, k + 1), -1, dtype=torch.int32)
    counts = torch.zeros(B, dtype=torch.int32)
    for b in range(B):
        s = 0 if b == 0 else int(cu[b - 1])
        e = min(int(cu[b]), draft.shape[0])
        n, acc, rej = 0, 0, False
        for p in range(s, e):
            d = int(draft[p])
            if d >= 0 and d == int(argmax[p]):
                out[b, n] = d
                n += 1
                acc += 1
            else:
                out[b, n] = int(argmax[p])
                n += 1
                rej = True
                break
        if not rej and s + acc < argmax.shape[0]:
            out[b, n] = int(argmax[s + acc])
        counts[b] = acc
    return out, counts


def emit(count, mask, draft, argmax, cu, k):
    B = mask.shape[0]
    out = torch.full((B, k + 1), -1, dtype=torch.int32)
    for b in range(B):
        s = 0 if b == 0 else int(cu[b - 1])
        c = int(count[b])
        for p in range(c):
            out[b, p] = int(draft[s + p])
        if mask[b, c] == 1:
            out[b, c] = int(argmax[s + c])
    return out


def test_random_batches_bit_exact():
    rng = np.random.default_rng(1234)
    for trial in range(200):
        B = int(rng.integers(1, 9))
        nd = [int(rng.integers(0, K + 1)) for _ in range(B)]
        g = torch.Generator().manual_seed(int(rng.integers(0, 10_000)))
        logits = torch.randn((B * (K + 1), 11), generator=g)
        rows = []
        for n in nd:
            d = torch.randint(0, 11, (K,), generator=g)
            d[n:] = -1
            rows.append(d)
        draft = torch.cat(rows)
        cu = torch.tensor(np.cumsum([K] * B), dtype=torch.int64)
        ref_out, ref_counts = torch_greedy(draft, logits[:draft.shape[0]], cu, K)
        am = logits[:draft.shape[0]].argmax(-1).numpy().astype(np.int64)
        count, mask = rejection_greedy_accept(draft.numpy().astype(np.int64), am, cu.numpy(), K)
        assert torch.equal(ref_counts, torch.as_tensor(count)), trial
        assert torch.equal(ref_out, emit(count, mask, draft.numpy(), am, cu.numpy(), K)), trial


def test_edges():
    am = np.full(K, 7, dtype=np.int64)
    cu = np.array([K], dtype=np.int64)
    c, m = rejection_greedy_accept(np.full(K, 7, dtype=np.int64), am, cu, K)
    assert int(c[0]) == K and int(m.sum()) == K + 1
    c, m = rejection_greedy_accept(np.full(K, 9, dtype=np.int64), am, cu, K)
    assert int(c[0]) == 0 and int(m.sum()) == 1
    d = np.full(K, 7, dtype=np.int64)
    d[2:] = -1
    c, m = rejection_greedy_accept(d, am, cu, K)
    assert int(c[0]) == 2 and int(m[0].sum()) == 3
    with pytest.raises(ValueError):
        rejection_greedy_accept(d[:3], am, cu, K)
