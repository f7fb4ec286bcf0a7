"""MXFP8 (W8A8, e4m3 with ue8m0 scales per 32) block-scaled tcgen05 GEMM (kind::mxf8f6f4) and its
activation quantiser against the fp32 PyTorch restatement."""
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _deswizzle(x_sf, rows, tile_rows, nblk):
    sf = x_sf.cpu()
    out = torch.zeros(rows, nblk, dtype=torch.uint8)
    for r in range(rows):
        t, i = r // tile_rows, r % tile_rows
        for b in range(nblk):
            out[r, b] = sf[t, b // 4, (i % 32) * 16 + (i // 32) * 4 + b % 4]
    return out


@pytest.mark.parametrize("rows,K,tile", [(70, 512, 64), (130, 1024, 128)])
def test_quant_act_matches_reference(rows, K, tile):
    torch.manual_seed(rows)
    x = (torch.randn(rows, K) * 3).to(torch.bfloat16)
    x[0, :32] = 0
    codes, scales = ref.mxfp8_quantize(x)
    xq, x_sf, a_sc = ops.mxfp8_quant_act(x.cuda(), tile)
    torch.cuda.synchronize()
    assert torch.equal(xq.cpu(), codes)
    assert torch.equal(_deswizzle(x_sf, rows, tile, K // 32), scales)
    assert torch.all(a_sc.cpu() == 1.0)


@pytest.mark.parametrize("M", [1, 64, 100, 192])
@pytest.mark.parametrize("N,K", [(384, 512), (1000, 2048)])
def test_mxfp8_linear_matches_fp32_oracle(M, N, K):
    torch.manual_seed(M + N + K)
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    codes, scales = ref.mxfp8_quantize(w)
    x = torch.randn(M, K).to(torch.bfloat16)
    want = ref.mxfp8_linear(x, codes, scales)
    got = ops.mxfp8_linear(x.cuda(), codes.cuda(), ops.mxfp8_scale_tiles(scales.cuda()), scales.cuda())
    torch.cuda.synchronize()
    err = (got.float().cpu() - want).abs().max().item()
    assert err <= 0.01 * want.abs().max().item() + 1e-3, err


def test_mxfp8_one_hot_reads_exact_products():
    """x = 3 e_k: each output is exactly 3 * w[n, k] after both quantisations (power-of-two scales)."""
    torch.manual_seed(2)
    N, K = 256, 256
    w = (torch.randn(N, K) * 0.05).to(torch.bfloat16)
    codes, scales = ref.mxfp8_quantize(w)
    x = torch.zeros(K, K, dtype=torch.bfloat16)
    x[torch.arange(K), torch.arange(K)] = 3.0
    want = ref.mxfp8_linear(x, codes, scales)
    got = ops.mxfp8_linear(x.cuda(), codes.cuda(), ops.mxfp8_scale_tiles(scales.cuda()), scales.cuda())
    torch.cuda.synchronize()
    assert torch.equal(got.float().cpu(), want.bfloat16().float())


def test_mxfp8_moe_experts_match_cpu_oracle():
    torch.manual_seed(5)
    E, H, F, T, k = 8, 256, 128, 40, 2
    w13 = (torch.randn(E * 2 * F, H) * 0.05).to(torch.bfloat16)
    w2 = (torch.randn(E * H, F) * 0.05).to(torch.bfloat16)
    q13, q2 = ref.mxfp8_quantize(w13), ref.mxfp8_quantize(w2)
    x = torch.randn(T, H).to(torch.bfloat16)
    ids = torch.stack([torch.randperm(E)[:k] for _ in range(T)]).int()
    wts = torch.rand(T, k).float()
    want = ops.moe_experts_mxfp8(x, ids, wts, q13, q2, E, F).float()
    cu = lambda q, r: (q[0].cuda(), q[1].cuda(), ops.mxfp8_scale_tiles(q[1].cuda(), r))
    got = ops.moe_experts_mxfp8(x.cuda(), ids.cuda(), wts.cuda(), cu(q13, 2 * F), cu(q2, H), E, F)
    torch.cuda.synchronize()
    err = (got.float().cpu() - want).abs().max().item()
    assert err <= 0.03 * want.abs().max().item() + 0.01, err
