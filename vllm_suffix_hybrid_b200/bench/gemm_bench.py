"""tcgen05 GEMM vs cuBLAS (torch.matmul) on the decode/verify GEMM shapes.

Times each shape with CUDA events after warm-up; between timed iterations a
256 MB buffer is rewritten so every iteration starts with a cold L2.
Reports microseconds, TFLOP/s and weight-stream GB/s per implementation.
Run: python -m vllm_suffix_hybrid_b200.bench.gemm_bench [--json]
"""
import argparse
import json

import torch

SHAPES = [  # (name, M, N, K) -- Llama-3-8B decode with a k=5 verify window over 64 rows
    ("qkv_m384", 384, 6144, 4096),
    ("o_m384", 384, 4096, 4096),
    ("gate_up_m384", 384, 28672, 4096),
    ("down_m384", 384, 4096, 14336),
    ("lm_head_m384", 384, 128256, 4096),
    ("qkv_m64", 64, 6144, 4096),
    ("gate_up_m64", 64, 28672, 4096),
    ("down_m64", 64, 4096, 14336),
    ("lm_head_m64", 64, 128256, 4096),
    ("square_4096", 4096, 4096, 4096),
]


def time_fn(fn, flush, iters=20, warmup=5):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    total = 0.0
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        e.synchronize()
        total += s.elapsed_time(e)
    return total / iters * 1e3  # us


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="", help="comma-separated shape names")
    ap.add_argument("--no-cublas", action="store_true")
    a = ap.parse_args()
    from vllm_suffix_hybrid_b200.ops.gemm import plan, tcgen05_linear

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    res = []
    only = set(filter(None, a.only.split(",")))
    for name, M, N, K in SHAPES:
        if only and name not in only:
            continue
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t_ours = time_fn(lambda: tcgen05_linear(x, w, y), flush, a.iters)
        t_lib = float("nan") if a.no_cublas else time_fn(lambda: torch.matmul(x, w.t(), out=y), flush, a.iters)
        ref = (x.float() @ w.float().t())
        tcgen05_linear(x, w, y)
        err = (y.float() - ref).abs().max().item()
        flops = 2.0 * M * N * K
        wbytes = N * K * 2
        r = {"shape": name, "M": M, "N": N, "K": K, "plan": list(plan(M, N, K)), "tcgen05_us": round(t_ours, 2),
             "cublas_us": round(t_lib, 2), "speedup": round(t_lib / t_ours, 3),
             "tcgen05_tflops": round(flops / t_ours / 1e6, 1), "tcgen05_weight_gbs": round(wbytes / t_ours / 1e3, 1),
             "max_abs_err": err}
        res.append(r)
        if not a.json:
            print(r)
    if a.json:
        print(json.dumps(res))


if __name__ == "__main__":
    main()
