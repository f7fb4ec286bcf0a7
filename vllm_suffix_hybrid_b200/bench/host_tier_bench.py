"""Host KV tier resolver cost: one layer's resolve per decode step at a config-3 shape.

B requests (a rank's share of config 3: 32 requests / attention DP 8), each with a 32k-token context in
host memory and k + 1 = 6 query tokens selecting top-2048 keys.  Each step keeps a fraction `--reuse` of the
previous step's keys (the rest are drawn anew from the context), so the steady-state miss rate is about
1 - reuse.  Timed with CUDA events around single resolve launches after warm-up; prints one JSON line with
microseconds per call, rows fetched per call and the host-link bandwidth that implies.

Run: python -m vllm_suffix_hybrid_b200.bench.host_tier_bench [--reuse 0.9] [--requests 4] [--ctx 32768]
"""
from __future__ import annotations

import argparse
import json

import numpy as np
import torch

from ..engine.host_tier import HostKVTier, hot_rows_for
from ..models.common import AttnMeta
from ..ops import mla_fp4_row_bytes


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--requests", type=int, default=4)
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--topk", type=int, default=2048)
    ap.add_argument("--reuse", type=float, default=0.9)
    ap.add_argument("--steps", type=int, default=20)
    a = ap.parse_args()
    B, W, K = a.requests, a.k + 1, a.topk
    row = mla_fp4_row_bytes(512, 64)
    nbl = a.ctx // 64 + 2
    H = hot_rows_for(a.k, K)
    tier = HostKVTier(1, B * nbl + 1, 64, (row,), torch.uint8, B + 1, H, a.ctx + 64, B * W, K, "cuda")
    bt = (torch.arange(B * nbl, dtype=torch.int32) + 1).view(B, nbl).cuda()
    slots = torch.arange(1, B + 1, device="cuda")
    tier.reset(slots)
    seq = torch.full((B,), a.ctx, dtype=torch.long, device="cuda")
    pos = (torch.arange(a.ctx - W, a.ctx).repeat(B)).cuda()
    meta = AttnMeta(positions=pos, slot_mapping=torch.full((B * W,), -1, dtype=torch.long, device="cuda"),
                    block_tables=bt, seq_lens=seq, q_start=(torch.arange(B + 1) * W).cuda(),
                    tile_req=torch.zeros(1, dtype=torch.int32), tile_row0=torch.zeros(1, dtype=torch.int32),
                    state_slots=slots, window=W)
    rng = np.random.default_rng(0)
    # per request a pool of keys; each step every token takes top-k keys from it, the pool drifting by 1 - reuse
    pools = [rng.choice(a.ctx - W, size=K, replace=False) for _ in range(B)]

    def next_topk():
        rows = []
        for b in range(B):
            keep = rng.random(K) < a.reuse
            pools[b] = np.where(keep, pools[b], rng.integers(0, a.ctx - W, K))
            for t in range(W):
                rows.append(np.sort(pools[b]) if t == 0 else np.roll(np.sort(pools[b]), t))
        return torch.tensor(np.stack(rows), dtype=torch.int32).cuda()

    layer = tier.layer(0)
    topks = [next_topk() for _ in range(a.steps + 3)]
    for tk in topks[:3]:
        layer.resolve(tk, meta)
    torch.cuda.synchronize()
    s0 = tier.stats.clone()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
    for i, tk in enumerate(topks[3:]):
        ev[i][0].record()
        layer.resolve(tk, meta)
        ev[i][1].record()
    torch.cuda.synchronize()
    tier.check()
    us = float(np.median([e0.elapsed_time(e1) * 1e3 for e0, e1 in ev]))
    hits, fetched = (tier.stats - s0).tolist()
    rows_per_call = fetched / a.steps
    print(json.dumps({"us_per_resolve": round(us, 2), "requests": B, "query_tokens": B * W, "topk": K, "hot_rows": H,
                      "reuse": a.reuse, "hit_rate": round(hits / max(hits + fetched, 1), 4),
                      "rows_fetched_per_call": round(rows_per_call, 1),
                      "host_gb_s": round(rows_per_call * row / us / 1e3, 2),
                      "device_bytes_per_layer": tier.device_bytes, "host_bytes_per_layer": tier.host_bytes}))


if __name__ == "__main__":
    main()
