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


def test_nvfp4_moe_experts_match_bf16_path():
    """Grouped NVFP4 experts == the bf16 grouped path run on the same (dequantised) weights."""
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
