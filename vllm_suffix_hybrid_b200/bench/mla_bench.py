"""MLA decode (+ DSA top-k) microbenchmark on the DeepSeek-V3.2 decode-verify shape.

Default: 32 requests x 6 query tokens (k = 5 verify), 128 heads, latent 512 + rope 64,
top-2048 keys per token out of an 8k context, paged 64-token blocks in shuffled order.
Device time from CUDA-graph replays (L2 flushed between iterations), FLOP/s against the
measured bf16 GEMM peak (MEASURED_PEAKS.json) and gathered latent bytes against HBM.
Run: python -m vllm_suffix_hybrid_b200.bench.mla_bench [--dense] [--once]
"""
import argparse
import json
import math
import os

import numpy as np
import torch


def peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["bf16_tflops"]), float(d["hbm_gbs"])
    except Exception:
        return 1590.0, 6650.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reqs", type=int, default=32)
    ap.add_argument("--q", type=int, default=6)
    ap.add_argument("--heads", type=int, default=128)
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--topk", type=int, default=2048)
    ap.add_argument("--dense", action="store_true")
    ap.add_argument("--fp4", action="store_true", help="NVFP4 latent cache rows instead of bf16")
    ap.add_argument("--nsplit", type=int, default=0)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true", help="two eager launches, no timing (for ncu)")
    ap.add_argument("--stamps", action="store_true", help="per-CTA cycle counters of the tcgen05 kernel")
    a = ap.parse_args()
    from vllm_suffix_hybrid_b200 import ops
    from vllm_suffix_hybrid_b200.bench.gemm_bench import time_fn

    C, V, bs = 576, 512, 64
    B, T = a.reqs, a.reqs * a.q
    nb = (a.ctx + bs - 1) // bs
    latent = (torch.randn(B * nb + 1, bs, C, device="cuda") * 0.5).to(torch.bfloat16)
    bt = (torch.randperm(B * nb, device="cuda") + 1).view(B, nb).int()
    seq = torch.full((B,), a.ctx, dtype=torch.long, device="cuda")
    qs = torch.arange(B + 1, dtype=torch.long, device="cuda") * a.q
    q = (torch.randn(T, a.heads, C, device="cuda") * 0.3).to(torch.bfloat16)
    topk = None
    K = a.ctx if a.dense else a.topk
    if not a.dense:
        g = torch.Generator(device="cuda").manual_seed(0)
        topk = torch.stack([torch.randperm(a.ctx - a.q, device="cuda", generator=g)[:K].sort().values
                            for _ in range(T)]).int()
    if a.fp4:  # same values written through the NVFP4 cache writer
        flat = latent.view(-1, C)
        packed = torch.zeros(latent.shape[0], bs, ops.mla_fp4_row_bytes(V, C - V), dtype=torch.uint8, device="cuda")
        ops.mla_cache_write(packed, flat[:, :V].contiguous(), flat[:, V:].contiguous(),
                            torch.arange(flat.shape[0], device="cuda"))
        latent = packed
    nsplit = a.nsplit or ops.mla_splits(T, a.heads, K)
    run = lambda: ops.mla_decode(q, latent, bt, seq, qs, 1.0 / math.sqrt(192), V, topk, nsplit)
    if a.stamps:
        ctas = T * (a.heads // 128) * 2 * nsplit
        st = torch.zeros(ctas * 8, dtype=torch.long, device="cuda")
        for _ in range(2):
            st.zero_()
            ops.mla_decode(q, latent, bt, seq, qs, 1.0 / math.sqrt(192), V, topk, nsplit, stamps=st)
        torch.cuda.synchronize()
        st = st.view(ctas, 8).double().cpu()
        names = ["prod_wait_free", "prod_issue", "mma_wait_keys", "mma_wait_p", "softmax_wait_s", "rescales",
                 "cta_cycles", "tiles"]
        print(json.dumps({"stamps_median": {n: float(st[:, i].median()) for i, n in enumerate(names)},
                          "stamps_max": {n: float(st[:, i].max()) for i, n in enumerate(names)}}))
        return
    if a.once:
        run()
        run()
        torch.cuda.synchronize()
        print(json.dumps({"once": True, "nsplit": nsplit}))
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    us = time_fn(run, flush, a.iters)
    flops = 2.0 * T * a.heads * K * (C + V)
    row_bytes = latent.shape[2] if a.fp4 else C * 2
    gathered = T * K * row_bytes  # latent rows read per token (requests' tokens share most of them through L2)
    tf, hbm = peaks()
    print(json.dumps({"us": round(us, 2), "tokens": T, "heads": a.heads, "keys_per_token": K, "dense": a.dense, "fp4_cache": a.fp4,
                      "nsplit": nsplit, "tflops": round(flops / us / 1e6, 1),
                      "frac_of_measured_bf16_peak": round(flops / us / 1e6 / tf, 3),
                      "gathered_gb_s": round(gathered / us / 1e3, 1)}))


if __name__ == "__main__":
    main()
