"""NVFP4 (ModelOpt layout) quantise / dequantise kernels against the fp32 PyTorch restatement."""
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(64, 128), (384, 7168), (1, 16)])
def test_quantize_matches_reference(shape):
    torch.manual_seed(0)
    w = (torch.randn(*shape) * 0.05).to(torch.bfloat16)
    g = ref.nvfp4_global_scale(w)
    p_ref, s_ref = ref.nvfp4_quantize(w, g)
    p, s, g2 = ops.nvfp4_quantize(w.cuda(), g.cuda())
    torch.cuda.synchronize()
    assert torch.equal(s.cpu().view(torch.uint8), s_ref.view(torch.uint8))
    assert torch.equal(p.cpu(), p_ref)


def test_dequantize_matches_reference():
    torch.manual_seed(1)
    w = (torch.randn(256, 512) * 0.02).to(torch.bfloat16)
    g = ref.nvfp4_global_scale(w)
    p, s = ref.nvfp4_quantize(w, g)
    want = ref.nvfp4_dequantize(p, s, g).float()
    got = ops.nvfp4_dequantize(p.cuda(), s.cuda(), g.cuda())
    torch.cuda.synchronize()
    torch.testing.assert_close(got.float().cpu(), want, rtol=1e-2, atol=1e-6)


@pytest.mark.parametrize("M", [1, 64, 200, 384])
@pytest.mark.parametrize("N,K", [(512, 256), (1000, 7168), (7168, 512)])
def test_nvfp4_linear_matches_dequantised(M, N, K):
    """W4A16 tcgen05 kernel vs an fp32 matmul with the dequantised weight."""
    torch.manual_seed(M + N + K)
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    g = ref.nvfp4_global_scale(w)
    p, s = ref.nvfp4_quantize(w, g)
    wd = ref.nvfp4_dequantize(p, s, g).float()
    x = torch.randn(M, K).to(torch.bfloat16)
    want = x.float() @ wd.t()
    got = ops.nvfp4_linear(x.cuda(), p.cuda(), s.cuda(), g.cuda())
    torch.cuda.synchronize()
    err = (got.float().cpu() - want).abs().max().item()
    assert err <= 0.02 * want.abs().max().item() + 0.02, err


def test_nvfp4_moe_experts_match_bf16_path(monkeypatch):
    """Grouped NVFP4 experts (W4A16 mode) == the bf16 grouped path run on the same (dequantised) weights."""
    monkeypatch.setenv("SH_NVFP4_ACT", "bf16")
    torch.manual_seed(3)
    E, H, F, T, k = 8, 256, 128, 40, 2
    w13 = (torch.randn(E * 2 * F, H) * 0.05).to(torch.bfloat16).cuda()
    w2 = (torch.randn(E * H, F) * 0.05).to(torch.bfloat16).cuda()

    def quant(w, rows):
        ps, ss, gs = [], [], []
        for e in range(E):
            p, s, g = ops.nvfp4_quantize(w[e * rows:(e + 1) * rows])
            ps.append(p), ss.append(s), gs.append(g.reshape(1).float())
        return torch.cat(ps), torch.cat(ss), torch.cat(gs)

    q13, q2 = quant(w13, 2 * F), quant(w2, H)
    d13 = torch.cat([ops.nvfp4_dequantize(q13[0][e * 2 * F:(e + 1) * 2 * F], q13[1][e * 2 * F:(e + 1) * 2 * F],
                                          q13[2][e:e + 1]) for e in range(E)])
    d2 = torch.cat([ops.nvfp4_dequantize(q2[0][e * H:(e + 1) * H], q2[1][e * H:(e + 1) * H], q2[2][e:e + 1])
                    for e in range(E)])
    x = torch.randn(T, H).to(torch.bfloat16).cuda()
    ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).int().cuda()
    wts = torch.rand(T, k).float().cuda()
    got = ops.moe_experts_nvfp4(x, ids, wts, q13, q2, E, F)
    want = ops.moe_experts(x, ids, wts, d13, d2, E, F)
    torch.cuda.synchronize()
    err = (got.float() - want.float()).abs().max().item()
    assert err <= 0.03 * want.float().abs().max().item() + 0.02, err


def test_nvfp4_linear_decodes_every_code_exactly():
    """One-hot activations read single dequantised weights back: every e2m1 code (the subnormal 0.5
    included) times every block scale must come out exact."""
    torch.manual_seed(5)
    N, K = 256, 128
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    w[0, :16] = torch.tensor([0.0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.0, -0.5, -1, -1.5, -2, -3, -4, -6]) * 0.01
    g = ref.nvfp4_global_scale(w)
    p, s = ref.nvfp4_quantize(w, g)
    want = ref.nvfp4_dequantize(p, s, torch.ones(1)).float()  # code * block scale (global applied below)
    x = torch.eye(K).to(torch.bfloat16)
    got = ops.nvfp4_linear(x.cuda(), p.cuda(), s.cuda(), torch.ones(1).cuda())
    torch.cuda.synchronize()
    assert torch.equal(got.float().cpu(), want.t()), (got.float().cpu() - want.t()).abs().max()


# ----------------------------------------------------------------------------- W4A4 (block-scaled MMA)
def _deswizzle(x_sf, rows, tile_rows, kb16, groups=None):
    """Scale tiles [tiles, kc4, 512] -> per-row scales [rows, kb16] (uint8)."""
    sf = x_sf.cpu()
    out = torch.zeros(rows, kb16, dtype=torch.uint8)
    ent = [(t * tile_rows, min(tile_rows, rows - t * tile_rows)) for t in range(-(-rows // tile_rows))] \
        if groups is None else [tuple(g[:2]) for g in groups]
    for t, (q0, n) in enumerate(ent):
        for i in range(n):
            for b in range(kb16):
                out[q0 + i, b] = sf[t, b // 4, (i % 32) * 16 + (i // 32) * 4 + b % 4]
    return out


@pytest.mark.parametrize("rows,K,tile", [(100, 1024, 64), (3, 320, 128), (130, 7168, 128)])
@pytest.mark.parametrize("static_g", [0.0, 37.5])
def test_quant_act_matches_reference(rows, K, tile, static_g):
    torch.manual_seed(rows + K)
    x = (torch.randn(rows, K) * 3).to(torch.bfloat16)
    x[0, :16] = 0  # an all-zero block
    pq, ps, pa = ref.nvfp4_quant_act(x, static_g)
    xq, x_sf, a_sc = ops.nvfp4_quant_act(x.cuda(), tile, static_g)
    torch.cuda.synchronize()
    assert torch.equal(xq.cpu(), pq)
    assert torch.equal(a_sc.cpu(), pa.float())
    assert torch.equal(_deswizzle(x_sf, rows, tile, K // 16), ps)


@pytest.mark.parametrize("rows,F,tile", [(100, 1024, 64), (37, 2048, 128)])
def test_quant_act_swiglu_fusion_equals_silu_mul_then_quant(rows, F, tile):
    """The quantiser's fused SwiGLU reads gate | up and must equal silu_mul followed by the plain quantiser."""
    torch.manual_seed(rows + F)
    gu = (torch.randn(rows, 2 * F) * 2).to(torch.bfloat16).cuda()
    xq, x_sf, a_sc = [t.clone() for t in ops.nvfp4_quant_act(ops.silu_mul(gu), tile)]
    fq, f_sf, f_sc = ops.nvfp4_quant_act(gu, tile, swiglu=True)
    torch.cuda.synchronize()
    assert torch.equal(fq[:rows], xq[:rows])
    assert torch.equal(f_sc[:rows], a_sc[:rows])
    assert torch.equal(_deswizzle(f_sf, rows, tile, F // 16), _deswizzle(x_sf, rows, tile, F // 16))


def test_gather_of_prequantised_rows_equals_quantising_the_gathered_rows():
    """Rows quantised once (the NVFP4 expert-parallel dispatch's linear layout) and gathered into the grouped
    W4A4 operand must equal quantising the gathered bf16 rows: codes, scale tiles and token scales."""
    torch.manual_seed(9)
    R, K = 50, 1024
    x = (torch.randn(R, K) * 2).to(torch.bfloat16)
    x[3] = 0  # a zero row
    codes, scales, ascale = ref.nvfp4_quant_act(x)
    groups = torch.tensor([[0, 40, 0, 0], [40, 30, 0, 0], [70, 37, 0, 0]], dtype=torch.int32).cuda()
    ngroups = torch.tensor([3], dtype=torch.int32).cuda()
    pairs = 107
    token = torch.randint(0, R, (pairs,), dtype=torch.int32)
    xq_r, sf_r, a_r = [t.clone() for t in ops.nvfp4_quant_act(x.cuda()[token.long().cuda()], 64, 0.0, groups,
                                                               ngroups)]
    xq, sf, a = ops.nvfp4_gather_act(codes.cuda(), scales.cuda(), ascale.float().cuda(), token.cuda(), groups, ngroups)
    torch.cuda.synchronize()
    assert torch.equal(xq[:pairs], xq_r[:pairs])
    assert torch.equal(a[:pairs], a_r[:pairs])
    assert torch.equal(sf[:3], sf_r[:3])


def test_scale_tiles_match_the_swizzled_layout():
    """nvfp4_scale_tiles == the 128x4 layout byte (row/128)*kb_pad*128 + (kb/4)*512 + (row%32)*16 +
    ((row/32)%4)*4 + kb%4 for K a multiple of 256 (reference: kernels/nvfp4_gemm.py sf_offset)."""
    torch.manual_seed(9)
    N, K = 300, 512
    s = torch.randint(0, 127, (N, K // 16), dtype=torch.uint8)
    tiles = ops.nvfp4_scale_tiles(s).reshape(-1)
    kb_pad = K // 16
    for row in range(N):
        for kb in range(kb_pad):
            off = (row // 128) * kb_pad * 128 + (kb // 4) * 512 + (row % 32) * 16 + ((row // 32) % 4) * 4 + kb % 4
            assert int(tiles[off]) == int(s[row, kb])


@pytest.mark.parametrize("M", [1, 16, 64, 100, 192])
@pytest.mark.parametrize("N,K", [(384, 512), (1000, 7168), (256, 320)])
def test_w4a4_linear_matches_fp32_oracle(M, N, K):
    """Block-scaled tcgen05 W4A4 GEMM vs the fp32 sum of dequantised products of the same codes."""
    torch.manual_seed(M * 7 + N + K)
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    g = ref.nvfp4_global_scale(w)
    p, s = ref.nvfp4_quantize(w, g)
    x = torch.randn(M, K).to(torch.bfloat16)
    want = ref.nvfp4_w4a4_linear(x, p, s, g)
    w_sf = ops.nvfp4_scale_tiles(s.cuda())
    got = ops.nvfp4_linear_w4a4(x.cuda(), p.cuda(), w_sf, s.cuda(), g.cuda())
    torch.cuda.synchronize()
    err = (got.float().cpu() - want).abs().max().item()
    assert err <= 0.01 * want.abs().max().item() + 1e-3, err


def test_w4a4_one_hot_reads_exact_products():
    """x = c * e_k for a code value c: every output is c * sx * w[n, k] with exact fp32 math, so the
    kernel's scale handling (both operands' e4m3 tiles in TMEM) is checked bit for bit."""
    torch.manual_seed(11)
    N, K = 256, 256
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    g = ref.nvfp4_global_scale(w)
    p, s = ref.nvfp4_quantize(w, g)
    x = torch.zeros(K, K, dtype=torch.bfloat16)
    x[torch.arange(K), torch.arange(K)] = 3.0
    want = ref.nvfp4_w4a4_linear(x, p, s, torch.ones(1))
    got = ops.nvfp4_linear_w4a4(x.cuda(), p.cuda(), ops.nvfp4_scale_tiles(s.cuda()), s.cuda(), torch.ones(1).cuda())
    torch.cuda.synchronize()
    assert torch.equal(got.float().cpu(), want.bfloat16().float())


def test_w4a4_moe_experts_match_cpu_oracle():
    torch.manual_seed(4)
    E, H, F, T, k = 8, 256, 128, 40, 2
    w13 = (torch.randn(E * 2 * F, H) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E * H, F) * 0.05).to(torch.bfloat16)

    def quant(w, rows):
        ps, ss, gs = [], [], []
        for e in range(E):
            g = ref.nvfp4_global_scale(w[e * rows:(e + 1) * rows])
            p, s = ref.nvfp4_quantize(w[e * rows:(e + 1) * rows], g)
            ps.append(p), ss.append(s), gs.append(g.reshape(1).float())
        return torch.cat(ps), torch.cat(ss), torch.cat(gs)

    q13, q2 = quant(w13, 2 * F), quant(w2, H)
    x = torch.randn(T, H).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).int()
    wts = torch.rand(T, k).float()
    want = ops.moe_experts_nvfp4(x, ids, wts, q13, q2, E, F).float()
    cu = lambda q, r: (q[0].cuda(), q[1].cuda(), q[2].cuda(), None, ops.nvfp4_scale_tiles(q[1].cuda(), r))
    got = ops.moe_experts_nvfp4(x.cuda(), ids.cuda(), wts.cuda(), cu(q13, 2 * F), cu(q2, H), E, F)
    torch.cuda.synchronize()
    err = (got.float().cpu() - want).abs().max().item()
    assert err <= 0.03 * want.abs().max().item() + 0.01, err


@pytest.mark.parametrize("splits", [2, 3, 5])
def test_w4a4_split_k_last_arriver_reduction(splits):
    """Forced split-K: the last split of each tile sums the partials in split order (matches the
    unsplit result to fp32 rounding) and leaves every ticket at zero for the next launch."""
    torch.manual_seed(21 + splits)
    M, N, K = 40, 520, 2560
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    g = ref.nvfp4_global_scale(w)
    p, s = ref.nvfp4_quantize(w, g)
    x = torch.randn(M, K).to(torch.bfloat16).cuda()
    pc, sc, gc = p.cuda(), s.cuda(), g.cuda().float()
    w_sf = ops.nvfp4_scale_tiles(sc)
    xq, x_sf, a_sc = [t.clone() for t in ops.nvfp4_quant_act(x, 64)]
    y1 = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ops.native().gemm_fp4mma(y1, xq, x_sf, a_sc, pc, w_sf, gc, 64)
    tiles = -(-N // 128) * -(-M // 64)
    ws = torch.empty(splits * tiles * 128 * 64, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(tiles, dtype=torch.int32, device="cuda")
    for _ in range(2):  # a second launch reuses the re-armed tickets
        ys = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        ops.native().gemm_fp4mma(ys, xq, x_sf, a_sc, pc, w_sf, gc, 64, splits=splits, ws=ws, counters=cnt)
        torch.cuda.synchronize()
        assert int(cnt.abs().sum()) == 0
        torch.testing.assert_close(ys.float(), y1.float(), rtol=2e-2, atol=2e-3)
    want = ref.nvfp4_w4a4_linear(x.cpu(), p, s, g)
    assert (ys.float().cpu() - want).abs().max().item() <= 0.01 * want.abs().max().item() + 1e-3


def test_screened_lm_head_on_gpu():
    """W4A4 screen + exact re-score of 64 candidates picks the bf16 head's greedy token (rows whose bf16
    maxima differ only by the fp32 summation order may flip; at most one here)."""
    from vllm_suffix_hybrid_b200.models.lm_head import ScreenedHead

    torch.manual_seed(12)
    V, H, M = 32000, 1024, 48
    w = (torch.randn(V, H, device="cuda") * 0.05).to(torch.bfloat16)
    x = torch.randn(M, H, device="cuda").to(torch.bfloat16)
    head = ScreenedHead(w)
    val, ids = head.best(x)
    want = (x.float() @ w.float().t()).bfloat16().float()
    torch.cuda.synchronize()
    assert int((ids != want.argmax(-1)).sum()) <= 1
    assert torch.allclose(val, want.max(-1).values, rtol=1e-2, atol=1e-3)
