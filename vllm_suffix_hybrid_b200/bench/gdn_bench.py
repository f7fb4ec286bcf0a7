"""Gated DeltaNet recurrent kernel and the fused draft-verification kernel: device microbenchmarks.

GDN (Qwen3-Next shape: 16 qk heads x 128, 32 v heads x 128): decode-verify windows (mode 1, k = 5: six
tokens per request after replaying the previous step's accepted records), prefill runs (mode 0) of the
recurrent kernel and of the chunked tensor-core prefill.
State bytes = requests x 32 heads x 128 x 128 x 4 (read + write per call).  spec_verify: greedy accept
+ commit of B windows.  Device time from CUDA-graph replays with the L2 flushed between iterations.
Run: python -m vllm_suffix_hybrid_b200.bench.gdn_bench [--once]
"""
import argparse
import json

import torch


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reqs", type=int, default=32)
    ap.add_argument("--prefill", type=int, default=1024, help="tokens per request of the prefill case")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true", help="one decode-window launch pair, no timing (for ncu)")
    ap.add_argument("--chunk-once", action="store_true", help="one chunked-prefill launch, no timing (for ncu)")
    a = ap.parse_args()
    from vllm_suffix_hybrid_b200 import ops
    from vllm_suffix_hybrid_b200.bench.gemm_bench import time_fn

    H, HV, K, W = 16, 32, 128, 6
    B = a.reqs
    dev = "cuda"
    slots = torch.arange(1, B + 1, device=dev)
    state = torch.zeros(B + 1, HV, K, K, device=dev)
    rec = (torch.zeros(B + 1, W, HV, K, device=dev), torch.zeros(B + 1, W, HV, K, device=dev),
           torch.zeros(B + 1, W, HV, device=dev), torch.zeros(B + 1, W, HV, device=dev))
    pending = torch.zeros(B + 2, dtype=torch.int32, device=dev)
    a_log = torch.randn(HV, device=dev) * 0.1
    dt_bias = torch.randn(HV, device=dev) * 0.1
    norm_w = torch.ones(K, device=dev, dtype=torch.bfloat16)

    def case(T, mode):
        qkv = (torch.randn(T, 2 * H * K + HV * K, device=dev) * 0.5).to(torch.bfloat16)
        z = (torch.randn(T, HV * K, device=dev)).to(torch.bfloat16)
        ba = (torch.randn(T, 2 * HV, device=dev)).to(torch.bfloat16)
        out = torch.empty(T, HV * K, device=dev, dtype=torch.bfloat16)
        qs = (torch.arange(B + 1, device=dev) * (T // B)).long()
        return lambda: ops.gdn_recurrent(qkv, z, ba, a_log, dt_bias, norm_w, state, rec, pending, slots, qs, out, H,
                                         HV, K, W, mode, 1e-6)

    dec = case(B * W, 1)
    pending[1:B + 1] = 3  # replay three accepted records per request before the window
    vd = torch.randint(0, 1000, (B, 5), device=dev)
    vt = torch.randint(0, 1000, (B, 6), device=dev)
    vt[:, :3] = vd[:, :3]
    seq = torch.zeros(B, dtype=torch.long, device=dev)
    o_t = torch.empty(B, 6, dtype=torch.long, device=dev)
    acc = torch.empty(B, dtype=torch.int32, device=dev)
    nxt = torch.empty(B, dtype=torch.long, device=dev)
    ver = lambda: ops.spec_verify(vd, vt, seq, o_t, acc, nxt)
    if a.chunk_once:  # one chunked-prefill launch (for ncu)
        T = B * a.prefill
        qkv = (torch.randn(T, 2 * H * K + HV * K, device=dev) * 0.5).to(torch.bfloat16)
        z = torch.randn(T, HV * K, device=dev).to(torch.bfloat16)
        ba = torch.randn(T, 2 * HV, device=dev).to(torch.bfloat16)
        out = torch.empty(T, HV * K, device=dev, dtype=torch.bfloat16)
        qs = (torch.arange(B + 1, device=dev) * a.prefill).long()
        ops.gdn_chunk_prefill(qkv, z, ba, a_log, dt_bias, norm_w, state, slots, qs, out, H, HV, K, 1e-6)
        torch.cuda.synchronize()
        print(json.dumps({"chunk_once": True}))
        return
    if a.once:
        for _ in range(2):
            dec()
            ver()
        torch.cuda.synchronize()
        print(json.dumps({"once": True}))
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    state_bytes = B * HV * K * K * 4 * 2
    us_dec = time_fn(dec, flush, a.iters)
    pre = case(B * a.prefill, 0)
    us_pre = time_fn(pre, flush, max(3, a.iters // 4))
    T = B * a.prefill
    qkv = (torch.randn(T, 2 * H * K + HV * K, device=dev) * 0.5).to(torch.bfloat16)
    z = torch.randn(T, HV * K, device=dev).to(torch.bfloat16)
    ba = torch.randn(T, 2 * HV, device=dev).to(torch.bfloat16)
    out = torch.empty(T, HV * K, device=dev, dtype=torch.bfloat16)
    qs = (torch.arange(B + 1, device=dev) * a.prefill).long()
    chunk = lambda: ops.gdn_chunk_prefill(qkv, z, ba, a_log, dt_bias, norm_w, state, slots, qs, out, H, HV, K, 1e-6)
    us_chunk = time_fn(chunk, flush, max(3, a.iters // 4))
    us_ver = time_fn(ver, flush, a.iters)
    print(json.dumps({"gdn_decode_window_us": round(us_dec, 2), "requests": B, "window": W,
                      "state_gb_s": round(state_bytes / us_dec / 1e3, 1),
                      "gdn_prefill_us": round(us_pre, 1), "prefill_tokens_per_request": a.prefill,
                      "prefill_tokens_per_s": round(B * a.prefill / us_pre * 1e6),
                      "gdn_chunk_prefill_us": round(us_chunk, 1),
                      "chunk_prefill_tokens_per_s": round(B * a.prefill / us_chunk * 1e6),
                      "spec_verify_us": round(us_ver, 2)}))


if __name__ == "__main__":
    main()
