"""tcgen05 GEMM vs a plain PyTorch fp32 matmul of the same bf16 operands."""
import pytest
import torch

from vllm_suffix_hybrid_b200 import ops
from vllm_suffix_hybrid_b200.ops import gemm

pytestmark = pytest.mark.gpu


def ref(x, w):
    return (x.float() @ w.float().t())


def check(y, x, w):
    want = ref(x, w)
    err = (y.float() - want).abs().max().item()
    scale = want.abs().max().item() + 1e-6
    assert err <= 0.02 * scale + 0.02, f"max err {err} (scale {scale})"


@pytest.mark.parametrize("M", [1, 7, 64, 100, 256, 384, 777])
@pytest.mark.parametrize("N,K", [(64, 64), (200, 256), (4096, 4096), (1000, 1024)])
def test_gemm_planned(M, N, K):
    torch.manual_seed(M + N + K)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    check(gemm.tcgen05_linear(x, w), x, w)


@pytest.mark.parametrize("swap", [False, True])
@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("splits", [1, 3])
def test_gemm_variants(swap, bn, splits):
    torch.manual_seed(bn + splits)
    M, N, K = (96, 640, 1536) if swap else (300, 520, 1536)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ws = torch.empty(splits * M * N, device="cuda", dtype=torch.float32) if splits > 1 else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.native().gemm_bf16(y, x, w, swap, bn, splits, ws, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    check(y, x, w)


def test_gemm_strided_input_and_graph_capture():
    x_full = torch.randn(64, 2 * 1024, device="cuda", dtype=torch.bfloat16)
    x = x_full[:, :1024]  # row stride 2048 elements (16-byte multiple)
    w = torch.randn(512, 1024, device="cuda", dtype=torch.bfloat16) * 0.05
    check(gemm.tcgen05_linear(x, w), x, w)
    y = torch.empty(64, 512, device="cuda", dtype=torch.bfloat16)
    gemm.tcgen05_linear(x, w, y)  # sizes any workspace eagerly before capture
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        gemm.tcgen05_linear(x, w, y)
    x_full.normal_()
    g.replay()
    torch.cuda.synchronize()
    check(y, x, w)


@pytest.mark.parametrize("swap", [False, True])
@pytest.mark.parametrize("bn", [128, 192, 256])
@pytest.mark.parametrize("splits", [1, 3])
@pytest.mark.parametrize("M,N,K", [(300, 520, 1536), (384, 6144, 4096), (96, 640, 1536), (1000, 136, 512)])
def test_gemm_pair_variants(swap, bn, splits, M, N, K):
    """CTA-pair (cta_group::2) kernel: partial and fully out-of-range half tiles, both orientations."""
    torch.manual_seed(bn + splits + M)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    y = torch.full((M, N), float("nan"), device="cuda", dtype=torch.bfloat16)
    ws = torch.empty(splits * M * N, device="cuda", dtype=torch.float32) if splits > 1 else None
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.native().gemm_bf16(y, x, w, swap, bn, splits, ws, err, True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    check(y, x, w)
