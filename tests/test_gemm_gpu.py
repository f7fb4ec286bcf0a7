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


SK_VARIANTS = [(64, 1), (128, 1), (192, 1), (256, 1), (192, 2), (256, 2)]


def _sk_buffers(M, N, ns, nsub, clusters):
    nt = ns * nsub
    tiles = -(-N // 256) * -(-M // nt)
    ws = torch.full((clusters * 4 * nt * 128,), float("nan"), device="cuda", dtype=torch.float32)
    cnt = torch.zeros(2 * tiles, device="cuda", dtype=torch.int32)
    return ws, cnt


@pytest.mark.parametrize("ns,nsub", SK_VARIANTS)
@pytest.mark.parametrize("M,N,K,clusters", [
    (384, 6144, 4096, 74),   # verify-size qkv: tiles cut into several pieces
    (64, 4096, 14336, 74),   # draft-size down: long K
    (300, 520, 1536, 74),    # ragged token and weight edges, pieces of partial tiles
    (37, 1000, 512, 3),      # few clusters: several whole tiles per cluster
    (200, 2056, 1024, 9),    # weight rows not a multiple of the 256-row tile
    (384, 28672, 1024, 74),  # 1.5 waves: split ranges span two tiles, a fix-up waits behind the next piece
])
def test_gemm_streamk(ns, nsub, M, N, K, clusters):
    """Stream-K CTA-pair kernel against fp32; output outside the problem untouched, counters left zero."""
    torch.manual_seed(ns + nsub + M + N)
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    y_full = torch.full((M + 5, N + 8), 7.0, device="cuda", dtype=torch.bfloat16)
    y = y_full[:M, :N]  # row stride N + 8: the TMA store must clip at the view's bounds
    ws, cnt = _sk_buffers(M, N, ns, nsub, clusters)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ops.native().gemm_bf16_sk(y, x, w, ns, nsub, clusters, ws, cnt, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(cnt.abs().sum().item()) == 0
    check(y, x, w)
    assert bool((y_full[M:] == 7.0).all()) and bool((y_full[:, N:] == 7.0).all())


def test_gemm_streamk_deterministic_and_graph():
    """Pieces are summed in cluster order: repeated calls and a graph replay agree bit for bit."""
    torch.manual_seed(5)
    M, N, K = 384, 4096, 14336
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
    ws, cnt = _sk_buffers(M, N, 192, 2, 74)
    y0 = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    ops.native().gemm_bf16_sk(y0, x, w, 192, 2, 74, ws, cnt)
    check(y0, x, w)
    y1 = torch.empty_like(y0)
    for _ in range(3):
        ops.native().gemm_bf16_sk(y1, x, w, 192, 2, 74, ws, cnt)
        torch.cuda.synchronize()
        assert torch.equal(y0, y1)
    g = torch.cuda.CUDAGraph()
    y2 = torch.empty_like(y0)
    with torch.cuda.graph(g):
        ops.native().gemm_bf16_sk(y2, x, w, 192, 2, 74, ws, cnt)
    for _ in range(2):
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y0, y2)
    assert int(cnt.abs().sum().item()) == 0


def test_planned_linears_use_no_library_gemm():
    """The default candidate list has no cuBLAS entry; the decode shapes plan onto tcgen05 kernels."""
    from vllm_suffix_hybrid_b200.ops.gemm import candidates

    for M, N, K in [(384, 28672, 4096), (64, 128256, 4096), (6, 4096, 4096)]:
        assert all(c.kind != "lib" for c in candidates(M, N, K))
