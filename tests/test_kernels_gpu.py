"""sm_100a kernels vs plain PyTorch fp32 statements of the same ops."""
import math

import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _need_cuda():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    ops.native()  # the extension must load on a GPU host
    torch.manual_seed(0)


def close(a, b, tol):
    err = (a.detach().float().cpu() - b.detach().float().cpu()).abs().max().item()
    assert err <= tol, f"max abs err {err} > {tol}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("hidden", [256, 4096, 7168])
def test_rms_norm(dtype, hidden):
    x = torch.randn(37, hidden, device="cuda", dtype=dtype)
    w = torch.randn(hidden, device="cuda", dtype=dtype)
    close(ops.rms_norm(x, w, 1e-5), ref.rms_norm(x.cpu().float(), w.cpu().float(), 1e-5), 0.05 if dtype != torch.float32 else 1e-4)


@pytest.mark.parametrize("hidden", [256, 4096, 2048])
def test_fused_add_rms_norm(hidden):
    x = torch.randn(19, hidden, device="cuda", dtype=torch.bfloat16)
    r = torch.randn(19, hidden, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(hidden, device="cuda", dtype=torch.bfloat16)
    x2, r2 = x.cpu().clone(), r.cpu().clone()
    ops.fused_add_rms_norm(x, r, w, 1e-6)
    ref.fused_add_rms_norm(x2, r2, w.cpu(), 1e-6)
    close(r, r2, 0.0)
    close(x, x2, 0.06)


def _paged_setup(q_lens, ctx_lens, hq, hk, d, bs=64, dtype=torch.bfloat16):
    B = len(q_lens)
    seq = [c + q for c, q in zip(ctx_lens, q_lens)]
    maxb = max((s + bs - 1) // bs for s in seq)
    nblocks = B * maxb + 1
    k_cache = torch.randn(nblocks, hk, bs, d, device="cuda", dtype=dtype)
    v_cache = torch.randn(nblocks, hk, bs, d, device="cuda", dtype=dtype)
    perm = torch.randperm(nblocks - 1)[: B * maxb] + 1
    bt = perm.view(B, maxb).int().cuda()
    qs = torch.tensor([0] + list(np.cumsum(q_lens)), dtype=torch.long, device="cuda")
    T = int(sum(q_lens))
    qkv = torch.randn(T, (hq + 2 * hk) * d, device="cuda", dtype=dtype)
    return k_cache, v_cache, bt, torch.tensor(seq, dtype=torch.long, device="cuda"), qs, qkv


@pytest.mark.parametrize("nsplit", [1, 3])
@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("shape", [
    ([6] * 5, [100, 63, 64, 1, 700]),  # verify windows, k = 5
    ([1] * 7, [5, 64, 129, 300, 2048, 0, 77]),  # plain decode
    ([130, 1, 64], [0, 40, 200]),  # prefill / chunked prefill
])
def test_paged_attention(d, shape, nsplit):
    q_lens, ctx = shape
    hq, hk = 8, 2
    kc, vc, bt, seq, qs, qkv = _paged_setup(q_lens, ctx, hq, hk, d)
    tr, t0 = ops.plan_attention_tiles(q_lens, hq // hk)
    out = torch.empty(qkv.shape[0], hq * d, device="cuda", dtype=torch.bfloat16)
    scale = 1.0 / math.sqrt(d)
    ops.paged_attention(out, qkv, kc, vc, bt, seq, qs, torch.tensor(tr, dtype=torch.int32, device="cuda"),
                        torch.tensor(t0, dtype=torch.int32, device="cuda"), hq, scale, nsplit,
                        min(64, max(q_lens) * (hq // hk)))
    q = qkv[:, : hq * d].reshape(-1, hq, d)
    want = ref.paged_attention(q.cpu().float(), kc.cpu().float(), vc.cpu().float(), bt.cpu(), seq.cpu(), qs.cpu(),
                               hq, scale)
    close(out.view(-1, hq, d).cpu(), want, 0.03)


def test_rope_kv_write():
    hq, hk, d, T = 8, 2, 128, 13
    qkv = torch.randn(T, (hq + 2 * hk) * d, device="cuda", dtype=torch.bfloat16)
    pos = torch.randint(0, 4000, (T,), device="cuda")
    cs = ref.rope_cos_sin(4096, d, 500000.0, device="cuda")
    kc = torch.zeros(8, hk, 64, d, device="cuda", dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    slots = torch.randperm(8 * 64, device="cuda")[:T]
    slots[3] = -1
    q2, kc2, vc2 = qkv.cpu().clone(), kc.cpu().clone(), vc.cpu().clone()
    ops.rope_kv_write(qkv, pos, cs, kc, vc, slots, hq, hk, d)
    ref.rope_kv_write(q2, pos.cpu(), cs.cpu(), kc2, vc2, slots.cpu(), hq, hk, d, d)
    close(qkv.cpu(), q2, 0.02)
    close(kc.cpu(), kc2, 0.02)
    close(vc.cpu(), vc2, 0.0)


def test_silu_mul_embedding_argmax():
    x = torch.randn(9, 2 * 1024, device="cuda", dtype=torch.bfloat16)
    close(ops.silu_mul(x), ref.silu_mul(x.cpu()), 0.02)
    table = torch.randn(1000, 256, device="cuda", dtype=torch.bfloat16)
    ids = torch.randint(0, 1000, (17,), device="cuda")
    close(ops.embedding(ids, table), table[ids], 0.0)
    logits = torch.randn(33, 128256, device="cuda", dtype=torch.bfloat16)
    logits[5, 77] = 100.0
    logits[6, 10] = logits[6, 20] = 100.0  # tie: first index wins
    got = ops.argmax(logits)
    assert torch.equal(got.cpu(), logits.float().cpu().argmax(-1))
    assert int(got[6]) == 10


def test_spec_verify_matches_reference():
    B, k = 64, 5
    g = torch.Generator().manual_seed(3)
    target = torch.randint(0, 4, (B, k + 1), generator=g)
    draft = torch.where(torch.rand(B, k, generator=g) < 0.7, target[:, :k], torch.randint(0, 4, (B, k), generator=g))
    draft[::7, 2] = -1
    seq = torch.randint(10, 100, (B,), generator=g)
    o_ref, a_ref, n_ref, s_ref = ref.spec_verify(draft, target, seq)
    d_c, t_c, s_c = draft.cuda(), target.cuda(), seq.cuda()
    out = torch.empty(B, k + 1, dtype=torch.long, device="cuda")
    acc = torch.empty(B, dtype=torch.int32, device="cuda")
    nxt = torch.empty(B, dtype=torch.long, device="cuda")
    ops.spec_verify(d_c, t_c, s_c, out, acc, nxt)
    assert torch.equal(out.cpu(), o_ref) and torch.equal(acc.cpu(), a_ref)
    assert torch.equal(nxt.cpu(), n_ref) and torch.equal(s_c.cpu(), s_ref)


@pytest.mark.parametrize("T,V,offset", [(1, 16032, 0), (384, 16032, 48096), (77, 1008, 5)])
def test_argmax_tp_single_rank_layout(T, V, offset):
    """The fused vocab-parallel argmax in a one-rank layout (keys and flags in this GPU's memory):
    global id = local first-occurrence argmax + the shard's vocab offset, over repeated calls."""
    torch.manual_seed(T + V)
    logits = torch.randn(T, V, device="cuda").to(torch.bfloat16)
    logits[0, 3] = 50.0
    logits[0, 7] = 50.0  # tie: the lower id wins
    keys = torch.zeros(2 * 1 * 512 * 2 + 160 * 8, dtype=torch.int32, device="cuda")
    base = keys.data_ptr()
    counters = torch.zeros(160, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(T, dtype=torch.int64, device="cuda")
    want = logits.float().argmax(1) + offset
    for _ in range(3):  # both key parities
        ops.native().argmax_tp(out, logits, [base], [base + 2 * 512 * 8], counters, err, 0, 512, offset, 64)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out, want)
    assert int(out[0].item()) == 3 + offset
