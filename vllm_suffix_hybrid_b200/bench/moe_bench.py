"""MoE router and grouped-expert pipeline on one GPU at a config-3 rank's shape.

Router: sigmoid group-limited top-8 over 256 experts (8 groups, top-4 groups, bias), `--tokens` rows.
Experts: this rank's 32 of the 256 experts (expert parallelism 8) in bf16, hidden 7168, expert FFN 2048;
the routed pairs that fall on other ranks' experts are skipped, as after an expert-parallel dispatch.
The expert pipeline is align (counting sort) -> gather -> grouped gate_up GEMM -> SwiGLU -> grouped down
GEMM -> weighted combine.  The expert pipeline is timed with CUDA events per launch (median over `--iters`,
256 MB L2 flush before each); the router, whose kernel is shorter than its host launch, is timed as 50
back-to-back launches between two events (device time per launch, logits L2-warm after the first).
`--once` runs each op twice and exits (for ncu captures).

Run: python -m vllm_suffix_hybrid_b200.bench.moe_bench [--tokens 192] [--once]
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from .. import ops


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=192)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--local", type=int, default=32)
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--ffn", type=int, default=2048)
    ap.add_argument("--k", type=int, default=8)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true")
    a = ap.parse_args()
    torch.manual_seed(0)
    T, E, El, H, F = a.tokens, a.experts, a.local, a.hidden, a.ffn
    logits = torch.randn(T, E, device="cuda", dtype=torch.float32)
    bias = torch.randn(E, device="cuda") * 0.1
    x = torch.randn(T, H, device="cuda", dtype=torch.bfloat16)
    w13 = torch.randn(El * 2 * F, H, device="cuda", dtype=torch.bfloat16) * 0.02
    w2 = torch.randn(El * H, F, device="cuda", dtype=torch.bfloat16) * 0.02
    out = torch.empty(T, H, device="cuda", dtype=torch.bfloat16)

    def route():
        return ops.moe_route(logits, a.k, sigmoid_grouped=True, bias=bias, n_groups=8, topk_groups=4)

    ids, w = route()
    ids_local = torch.where(ids < El, ids, torch.full_like(ids, -1))  # this rank's experts only

    def experts():
        return ops.moe_experts(x, ids_local, w, w13, w2, El, F, out=out)

    if a.once:
        for _ in range(2):
            route()
            experts()
        torch.cuda.synchronize()
        print(json.dumps({"once": True}))
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def time_us(fn):
        for _ in range(3):
            fn()
        ts = []
        for _ in range(a.iters):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3)
        return float(np.median(ts))

    for _ in range(3):
        route()
    r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ids_buf = torch.empty(T, a.k, dtype=torch.int32, device="cuda")
    w_buf = torch.empty(T, a.k, dtype=torch.float32, device="cuda")
    lib = ops.native()
    torch.cuda.synchronize()
    r0.record()
    for _ in range(50):
        lib.moe_route(logits, bias, ids_buf, w_buf, a.k, True, 8, 4, True, 1.0)
    r1.record()
    torch.cuda.synchronize()
    t_route = r0.elapsed_time(r1) * 1e3 / 50
    t_exp = time_us(experts)
    pairs = int((ids_local >= 0).sum())
    flops = 2 * pairs * (2 * F * H + H * F)
    touched = int(torch.unique(ids_local[ids_local >= 0]).numel())
    wbytes = touched * (2 * F * H + H * F) * 2
    print(json.dumps({"tokens": T, "local_pairs": pairs, "experts_touched": touched, "route_us": round(t_route, 2),
                      "experts_us": round(t_exp, 2), "experts_tflops": round(flops / t_exp / 1e6, 1),
                      "expert_weight_gb_s": round(wbytes / t_exp / 1e3, 1)}))


if __name__ == "__main__":
    main()
