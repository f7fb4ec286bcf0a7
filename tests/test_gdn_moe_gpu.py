"""Gated DeltaNet and MoE kernels vs the plain PyTorch fp32 statements."""
import numpy as np
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _gdn_inputs(T, H, HV, K, seed):
    g = torch.Generator().manual_seed(seed)
    C = 2 * H * K + HV * K
    x = torch.randn(T, C + HV * K, generator=g).to(torch.bfloat16)
    ba = torch.randn(T, 2 * HV, generator=g).to(torch.bfloat16)
    w = torch.randn(C, 4, generator=g) * 0.5
    a_log = torch.log(torch.rand(HV, generator=g) * 8 + 1)
    dt = torch.full((HV,), 0.5)
    nw = (torch.rand(K, generator=g) + 0.5).to(torch.bfloat16)
    return x, ba, w, a_log, dt, nw, C


def _run(dev, x, ba, w, a_log, dt, nw, C, H, HV, K, slots, q_start, W, mode, cache, pending):
    T = x.shape[0]
    y = torch.empty(T, C, dtype=torch.bfloat16, device=dev)
    ops.gdn_conv(x.to(dev), w.to(dev), y, cache["conv"], cache["rx"], pending, slots, q_start, W, mode)
    out = torch.empty(T, HV * K, dtype=torch.bfloat16, device=dev)
    ops.gdn_recurrent(y, x.to(dev)[:, C:], ba.to(dev), a_log.to(dev), dt.to(dev), nw.to(dev), cache["S"],
                      (cache["rk"], cache["rv"], cache["rg"], cache["rb"]), pending, slots, q_start, out, H, HV, K,
                      W, mode, 1e-6)
    return y, out


def _cache(dev, slots, W, C, HV, K):
    f = dict(dtype=torch.float32, device=dev)
    return dict(S=torch.zeros(slots, HV, K, K, **f), conv=torch.zeros(slots, C, 3, **f),
                rx=torch.zeros(slots, W, C, **f), rk=torch.zeros(slots, W, HV, K, **f),
                rv=torch.zeros(slots, W, HV, K, **f), rg=torch.zeros(slots, W, HV, **f),
                rb=torch.zeros(slots, W, HV, **f))


@pytest.mark.parametrize("K,W,lens", [(64, 4, [11, 5]), (128, 4, [11, 5]), (128, 9, [37, 17]), (32, 6, [3, 9])])
def test_gdn_prefill_then_windows_match_reference(K, W, lens):
    """Prefill over several token chunks, then verify windows whose replayed records span chunks."""
    H, HV = 2, 4
    caches = {d: _cache(d, 3, W, 2 * H * K + HV * K, HV, K) for d in ("cpu", "cuda")}
    pend = {d: torch.zeros(3, dtype=torch.int32, device=d) for d in ("cpu", "cuda")}
    slots = {d: torch.tensor([2, 1], device=d) for d in ("cpu", "cuda")}
    # prefill
    x, ba, w, a_log, dt, nw, C = _gdn_inputs(sum(lens), H, HV, K, 0)
    qs = {d: torch.tensor([0, lens[0], sum(lens)], device=d) for d in ("cpu", "cuda")}
    outs = {d: _run(d, x, ba, w, a_log, dt, nw, C, H, HV, K, slots[d], qs[d], W, 0, caches[d], pend[d])
            for d in ("cpu", "cuda")}
    assert (outs["cuda"][1].float().cpu() - outs["cpu"][1].float()).abs().max() < 0.05
    # three verify windows with varying accepted counts
    for step, acc in enumerate([[min(2, W - 1), 0], [W - 1, 1], [0, W - 1]]):
        x, ba, *_ = _gdn_inputs(2 * W, H, HV, K, 10 + step)
        qs = {d: torch.tensor([0, W, 2 * W], device=d) for d in ("cpu", "cuda")}
        outs = {d: _run(d, x, ba, w, a_log, dt, nw, C, H, HV, K, slots[d], qs[d], W, 1, caches[d], pend[d])
                for d in ("cpu", "cuda")}
        err = (outs["cuda"][1].float().cpu() - outs["cpu"][1].float()).abs().max().item()
        assert err < 0.06, (step, err)
        for d in ("cpu", "cuda"):
            pend[d][2], pend[d][1] = acc[0] + 1, acc[1] + 1
    assert (caches["cuda"]["S"].cpu() - caches["cpu"]["S"]).abs().max() < 1e-2


@pytest.mark.parametrize("lens", [[150, 64, 7], [1, 200, 0, 65]])
def test_gdn_chunk_prefill_matches_recurrence(lens):
    """Chunked tensor-core prefill (64-token WY form, bf16 products) vs the fp32 recurrence on the CPU."""
    H, HV, K, W = 2, 4, 128, 4
    C = 2 * H * K + HV * K
    nreq = len(lens)
    x, ba, w, a_log, dt, nw, _ = _gdn_inputs(sum(lens), H, HV, K, 3)
    g = torch.Generator().manual_seed(5)
    qkv = (torch.randn(sum(lens), C, generator=g) * 0.7).to(torch.bfloat16)
    z = x[:, C:]
    qs = torch.tensor([0] + list(np.cumsum(lens)))
    slots = torch.arange(1, nreq + 1)
    st_c = torch.full((nreq + 1, HV, K, K), 7.0)
    out_c = torch.zeros(sum(lens), HV * K, dtype=torch.bfloat16)
    ops.gdn_chunk_prefill(qkv, z, ba, a_log, dt, nw, st_c, slots, qs, out_c, H, HV, K, 1e-6)
    dev = "cuda"
    st_g = torch.full((nreq + 1, HV, K, K), 7.0, device=dev)
    out_g = torch.zeros(sum(lens), HV * K, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    zg = x.to(dev)[:, C:]
    assert ops.gdn_chunk_ok(qkv.to(dev), zg, out_g, K)
    ops.gdn_chunk_prefill(qkv.to(dev), zg, ba.to(dev), a_log.to(dev), dt.to(dev), nw.to(dev), st_g, slots.to(dev),
                          qs.to(dev), out_g, H, HV, K, 1e-6, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    o_ref, o_got = out_c.float(), out_g.float().cpu()
    scale = o_ref.abs().max().item()
    assert (o_got - o_ref).abs().max().item() < 0.03 * scale, (o_got - o_ref).abs().max().item() / scale
    assert (o_got - o_ref).abs().mean().item() < 0.004 * scale
    s_ref, s_got = st_c, st_g.cpu()
    assert torch.equal(s_got[0], s_ref[0])  # untouched slot
    assert (s_got - s_ref).abs().max().item() < 0.03 * s_ref[1:].abs().max().item()


@pytest.mark.parametrize("grouped,E,k,groups,topg", [
    (False, 64, 6, 1, 1), (True, 64, 6, 8, 3),  # block path (8 experts per group)
    (True, 256, 8, 8, 4),                        # warp path: DeepSeek-V3 router
    (True, 384, 8, 1, 1),                        # warp path: Kimi-K2 (no group limit)
    (False, 512, 10, 1, 1),                      # warp path: Qwen3-Next softmax router
])
def test_moe_route(grouped, E, k, groups, topg):
    """The GPU router (one warp per token where E % 32 == 0, E <= 512 and 32 experts per group, else one
    block) picks the CPU statement's experts with its weights."""
    torch.manual_seed(E + k)
    T = 37
    logits = torch.randn(T, E)
    logits[3, 5] = logits[3, 9]  # an exact tie: the lower expert index is taken first
    bias = torch.randn(E) * 0.1 if grouped else None
    ids_c, w_c = ops.moe_route(logits, k, grouped, bias, groups, topg, True, 2.5)
    ids_g, w_g = ops.moe_route(logits.cuda(), k, grouped, bias.cuda() if grouped else None, groups, topg, True,
                               2.5)
    ids_b, w_b = ops.moe_route(logits.cuda().to(torch.bfloat16), k, grouped, bias.cuda() if grouped else None,
                               groups, topg, True, 2.5)
    assert bool((ids_b >= 0).all()) and bool((ids_b < E).all())
    assert torch.equal(ids_g.cpu().sort(-1).values, ids_c.sort(-1).values)
    o_c = w_c.gather(1, ids_c.long().argsort(-1))
    o_g = w_g.cpu().gather(1, ids_g.cpu().long().argsort(-1))
    assert (o_c - o_g).abs().max() < 1e-4


@pytest.mark.parametrize("T,E,k,F,H", [(384, 64, 8, 128, 256), (7, 16, 4, 64, 128), (200, 512, 10, 64, 128)])
def test_moe_experts_grouped_gemm(T, E, k, F, H):
    torch.manual_seed(T + E)
    x = torch.randn(T, H).to(torch.bfloat16)
    logits = torch.randn(T, E)
    ids, w = ops.moe_route(logits, k)
    w13 = (torch.randn(E * 2 * F, H) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E * H, F) * 0.05).to(torch.bfloat16)
    want = ops.moe_experts(x, ids, w, w13, w2, E, F)
    got = ops.moe_experts(x.cuda(), ids.cuda(), w.cuda(), w13.cuda(), w2.cuda(), E, F)
    torch.cuda.synchronize()
    err = (got.float().cpu() - want.float()).abs().max().item()
    assert err < 0.03 * want.float().abs().max().item() + 0.01, err
