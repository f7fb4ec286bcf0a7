"""Paged attention microbenchmark on the decode-verify shape.

Default: 64 requests x (2048 context + 6 verify tokens), 32 q heads / 8 kv
heads x 128 (Llama-3-8B), paged 64-token blocks in shuffled order.  The KV
working set (~550 MB) exceeds the 126 MB L2, so timed iterations start cold.
Reports microseconds, bytes of K/V streamed and the achieved fraction of the
measured HBM copy bandwidth (MEASURED_PEAKS.json, else 6450 GB/s).
Run: python -m vllm_suffix_hybrid_b200.bench.attn_bench [--iters N]
"""
import argparse
import json
import math
import os

import torch


def peak_gbs():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        return float(json.load(open(p))["hbm_gbs"])
    except Exception:
        return 6450.0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=2048)
    ap.add_argument("--q", type=int, default=6)
    ap.add_argument("--hq", type=int, default=32)
    ap.add_argument("--hk", type=int, default=8)
    ap.add_argument("--d", type=int, default=128)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--nsplit", type=int, default=0, help="0: framework default")
    a = ap.parse_args()
    from vllm_suffix_hybrid_b200 import ops

    B, bs = a.batch, 64
    seq = a.ctx + a.q
    nb_req = (seq + bs - 1) // bs
    nblocks = B * nb_req + 1
    kc = torch.randn(nblocks, a.hk, bs, a.d, device="cuda", dtype=torch.bfloat16)
    vc = torch.randn_like(kc)
    bt = (torch.randperm(nblocks - 1, device="cuda")[: B * nb_req] + 1).view(B, nb_req).int()
    T = B * a.q
    qkv = torch.randn(T, (a.hq + 2 * a.hk) * a.d, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(T, a.hq * a.d, device="cuda", dtype=torch.bfloat16)
    seq_lens = torch.full((B,), seq, device="cuda", dtype=torch.long)
    qs = torch.arange(B + 1, device="cuda", dtype=torch.long) * a.q
    tr, t0 = ops.plan_attention_tiles([a.q] * B, a.hq // a.hk)
    tr = torch.tensor(tr, dtype=torch.int32, device="cuda")
    t0 = torch.tensor(t0, dtype=torch.int32, device="cuda")
    nsplit = a.nsplit or ops.attention_splits(tr.numel(), a.hk, nb_req)
    max_rows = min(64, a.q * a.hq // a.hk)

    def run():
        ops.paged_attention(out, qkv, kc, vc, bt, seq_lens, qs, tr, t0, a.hq, 1.0 / math.sqrt(a.d), nsplit, max_rows)

    for _ in range(3):
        run()
    torch.cuda.synchronize()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    tot = 0.0
    for _ in range(a.iters):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        run()
        e.record()
        e.synchronize()
        tot += s.elapsed_time(e)
    us = tot / a.iters * 1e3
    kv_bytes = 2 * B * seq * a.hk * a.d * 2
    gbs = kv_bytes / us / 1e3
    print(json.dumps({"us": round(us, 2), "kv_bytes": kv_bytes, "gbs": round(gbs, 1),
                      "frac_of_measured_hbm": round(gbs / peak_gbs(), 3), "nsplit": nsplit, "max_rows": max_rows,
                      "batch": B, "ctx": a.ctx, "q": a.q, "hq": a.hq, "hk": a.hk, "d": a.d}))


if __name__ == "__main__":
    main()
