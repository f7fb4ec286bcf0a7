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
