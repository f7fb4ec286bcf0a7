"""DSA lightning-indexer microbenchmark on the DeepSeek-V3.2 decode-verify shape.

Default: 32 requests x 6 query rows (k = 5 verify), 64 index heads x 128, a 32k-key context per request in
shuffled 64-key fp8 pages (132 B per key), top-2048 per row.  Times the query quantisation, the tcgen05
scoring kernel and the top-k select from CUDA-graph replays with L2 flushed between iterations, and reports
the key bytes against the measured HBM copy bandwidth (MEASURED_PEAKS.json) and the fp8 MMA work.
Run: python -m vllm_suffix_hybrid_b200.bench.dsa_bench [--ctx 32768] [--once]
"""
import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reqs", type=int, default=32)
    ap.add_argument("--q", type=int, default=6)
    ap.add_argument("--heads", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--topk", type=int, default=2048)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true", help="two eager launches, no timing (for ncu)")
    a = ap.parse_args()
    from vllm_suffix_hybrid_b200 import ops
    from vllm_suffix_hybrid_b200.bench.gemm_bench import time_fn
    from vllm_suffix_hybrid_b200.bench.mla_bench import peaks

    B, T, IH = a.reqs, a.reqs * a.q, a.heads
    nb = (a.ctx + 63) // 64
    pages = B * nb + 1
    cache = ops.dsa_cache_alloc(pages, 64, "cuda")
    bt = (torch.randperm(B * nb, device="cuda") + 1).view(B, nb).int()
    pos = torch.arange(a.ctx, device="cuda")
    for b in range(B):  # keys through the cache writer
        k = (torch.randn(a.ctx, 128, device="cuda") * 0.5).to(torch.bfloat16)
        ops.dsa_cache_write(cache, k, bt[b, pos // 64].long() * 64 + pos % 64)
    seq = torch.full((B,), a.ctx, dtype=torch.long, device="cuda")
    qs = torch.arange(B + 1, dtype=torch.long, device="cuda") * a.q
    qi = (torch.randn(T, IH, 128, device="cuda") * 0.3).to(torch.bfloat16)
    w = torch.randn(T, IH, device="cuda")
    if a.once:
        for _ in range(2):
            ops.dsa_topk(qi, w, cache, bt, seq, qs, a.topk)
        torch.cuda.synchronize()
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ws = ops._dsa_ws(qi.device, T, IH, bt.shape[1] * 64)
    q8, wq, lg = ws["q8"][:T], ws["wq"][:T], ws["logits"][:T]
    ops.native().dsa_quant_q(q8, wq, qi, w)
    sms = ops._num_sms(qi.device)
    out = torch.empty(T, a.topk, dtype=torch.int32, device="cuda")
    t_all = time_fn(lambda: ops.dsa_topk(qi, w, cache, bt, seq, qs, a.topk), flush, a.iters)
    t_score = time_fn(lambda: ops.native().dsa_index(out, lg, q8, wq, cache, bt, seq, qs, sms, ws["err"], True),
                      flush, a.iters)
    t_quant = time_fn(lambda: ops.native().dsa_quant_q(q8, wq, qi, w), flush, a.iters)
    tflops, hbm = peaks()
    key_bytes = B * a.ctx * 132
    # per key and row: IH x 128 fp8 MACs (causal rows see slightly fewer keys)
    flops = 2.0 * T * a.ctx * IH * 128
    assert ws["err"].item() == 0, ws["err"].item()
    print(json.dumps({
        "bench": "dsa_indexer", "reqs": B, "rows_per_req": a.q, "heads": IH, "ctx": a.ctx, "topk": a.topk,
        "us_total": round(t_all, 2), "us_score": round(t_score, 2), "us_quant": round(t_quant, 2),
        "us_select": round(t_all - t_score - t_quant, 2),
        "key_MB": round(key_bytes / 1e6, 1),
        "score_hbm_frac_of_measured": round(key_bytes / (t_score * 1e-6) / (hbm * 1e9), 3),
        "total_hbm_frac_of_measured": round(key_bytes / (t_all * 1e-6) / (hbm * 1e9), 3),
        "score_fp8_tflops": round(flops / (t_score * 1e-6) / 1e12, 1),
        "score_fp8_frac_of_2x_bf16_measured": round(flops / (t_score * 1e-6) / (2 * tflops * 1e12), 3),
    }))


if __name__ == "__main__":
    main()
