"""tcgen05 GEMM vs cuBLAS (torch.matmul) on the decode/verify GEMM shapes.

Times each shape on the device from CUDA-graph replays (no host launch cost in
the number); between iterations a 256 MB buffer is rewritten so every
iteration starts with a cold L2.
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
    ("o_m64", 64, 4096, 4096),
    ("fc_m64", 64, 4096, 8192),  # EAGLE head input projection [embedding | hidden] -> hidden
    ("gate_up_m64", 64, 28672, 4096),
    ("down_m64", 64, 4096, 14336),
    ("lm_head_m64", 64, 128256, 4096),
    ("square_4096", 4096, 4096, 4096),
]


def time_fn(fn, flush, iters=20, warmup=5):
    """Device time of fn in microseconds, free of host launch cost.

    Captures `iters` x (L2 flush, fn) in one CUDA graph and `iters` x (flush)
    in another, replays both and returns the difference per iteration: what
    the kernels cost when replayed from a graph, as in the decode step.
    """
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    g1, g0 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g1):
        for _ in range(iters):
            flush.zero_()
            fn()
    with torch.cuda.graph(g0):
        for _ in range(iters):
            flush.zero_()

    def run(g):
        g.replay()
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(3):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            g.replay()
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        return best

    return max(run(g1) - run(g0), 0.0) / iters * 1e3  # us


def sweep(name, x, w, y, flush, iters):
    """Every candidate configuration of the autotuner on one shape (cuBLAS included)."""
    from vllm_suffix_hybrid_b200.ops.gemm import LIB, _runner, candidates

    M, K = x.shape
    N = w.shape[0]
    rows = []
    for cfg in [LIB] + [c for c in candidates(M, N, K) if c.kind != "lib"]:
        fn = _runner(cfg, x, w, y)
        try:
            fn()
        except RuntimeError:
            continue
        rows.append((time_fn(fn, flush, iters, 2), cfg))
    rows.sort(key=lambda r: r[0])
    print(json.dumps({"sweep": name, "M": M, "N": N, "K": K,
                      "cublas_us": round(next(t for t, c in rows if c.kind == "lib"), 2),
                      "best": [dict(us=round(t, 2), **c._asdict()) for t, c in rows[:8]]}), flush=True)


NVFP4_SHAPES = [  # (name, M, N, K): DeepSeek-V3-style decode projections and one expert
    ("q_b_m192", 192, 24576, 1536),
    ("o_m192", 192, 7168, 16384),
    ("expert_gate_up_m64", 64, 4096, 7168),
    ("expert_down_m64", 64, 7168, 2048),
    ("dense_gate_up_m192", 192, 36864, 7168),
    ("one_kblock_m64", 64, 4096, 256),  # launch + prologue + epilogue floor
]


def nvfp4_main(a):
    from vllm_suffix_hybrid_b200 import ops
    from vllm_suffix_hybrid_b200.ops.gemm import tcgen05_linear

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    only = set(filter(None, a.only.split(",")))
    for name, M, N, K in NVFP4_SHAPES:
        if only and name not in only:
            continue
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = (torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02)
        p, s, g = ops.nvfp4_quantize(w)
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        w_sf = ops.nvfp4_scale_tiles(s)
        run = lambda: ops.nvfp4_linear(x, p, s, g, out=y)
        run44 = lambda: ops.nvfp4_linear_w4a4(x, p, w_sf, s, g, out=y)
        if a.once:
            if a.mxfp8:
                c8, s8 = ops.mxfp8_quantize(w)
                t8sf = ops.mxfp8_scale_tiles(s8)
                run8 = lambda: ops.mxfp8_linear(x, c8, t8sf, s8, out=y)
                run8()
                run8()
            else:
                (run44 if a.w4a4 else run)()
                (run44 if a.w4a4 else run)()
            torch.cuda.synchronize()
            print(json.dumps({"once": name, "w4a4": bool(a.w4a4), "mxfp8": bool(a.mxfp8)}))
            continue
        if a.stamps:  # per-CTA timings of the W4A4 kernel at 1, 2, 4 and 8 K splits (cold L2)
            from vllm_suffix_hybrid_b200.ops.gemm import workspace
            bn44 = 64 if M <= 64 else 128
            xq, x_sf, a_sc = ops.nvfp4_quant_act(x, bn44)
            gsc = g.float().reshape(-1)
            nsm = torch.cuda.get_device_properties(0).multi_processor_count
            ntile = -(-N // 128) * -(-M // bn44)
            wsp = workspace(x.device, 8 * ntile * 128 * bn44)
            cnt = ops.split_tickets(x.device, ntile)
            keys = ["setup", "pdl_wait", "first_stage", "first_acc", "acc_waits", "split_part", "store", "cta"]
            for sp in (1, 2, 4, 8):
                st = torch.zeros(nsm * 8, dtype=torch.long, device="cuda")
                for _ in range(3):
                    flush.zero_()
                    st.zero_()
                    ops.native().gemm_fp4mma(y, xq, x_sf, a_sc, p, w_sf, gsc, bn44, splits=sp, ws=wsp, counters=cnt,
                                             stamps=st)
                torch.cuda.synchronize()
                v = st.view(nsm, 8).cpu()
                used = v[:, 7] > 0
                print(json.dumps({"stamps": name, "splits": sp, "ctas": int(used.sum()),
                                  "median_ns": dict(zip(keys, v[used].median(0).values.tolist())),
                                  "max_ns": dict(zip(keys, v[used].max(0).values.tolist()))}))
            continue
        t4 = time_fn(run, flush, a.iters)
        t44 = time_fn(run44, flush, a.iters)  # includes the activation quantiser launch
        bn44 = 64 if M <= 64 else 128
        xq, x_sf, a_sc = ops.nvfp4_quant_act(x, bn44)
        xq, x_sf, a_sc = xq.clone(), x_sf.clone(), a_sc.clone()
        tq = time_fn(lambda: ops.nvfp4_quant_act(x, bn44), flush, a.iters)
        gsc = g.float().reshape(-1)
        t_g1 = time_fn(lambda: ops.native().gemm_fp4mma(y, xq, x_sf, a_sc, p, w_sf, gsc, bn44), flush, a.iters)
        from vllm_suffix_hybrid_b200.ops.gemm import workspace
        ntile = -(-N // 128) * -(-M // bn44)
        wsp = workspace(x.device, 8 * ntile * 128 * bn44)
        cnt = ops.split_tickets(x.device, ntile)
        t_split = {sp: round(time_fn(lambda: ops.native().gemm_fp4mma(y, xq, x_sf, a_sc, p, w_sf, gsc, bn44,
                                                                      splits=sp, ws=wsp, counters=cnt),
                                     flush, a.iters), 2)
                   for sp in (2, 4, 8)}
        wd = ops.nvfp4_dequantize(p, s, g)
        c8, s8 = ops.mxfp8_quantize(w)
        t8sf = ops.mxfp8_scale_tiles(s8)
        t8 = time_fn(lambda: ops.mxfp8_linear(x, c8, t8sf, s8, out=y), flush, a.iters)
        t16 = time_fn(lambda: tcgen05_linear(x, wd, y), flush, a.iters)
        tlib = time_fn(lambda: torch.matmul(x, wd.t(), out=y), flush, a.iters)
        ref = x.float() @ wd.float().t()
        err = (ops.nvfp4_linear(x, p, s, g).float() - ref).abs().max().item()
        ref44 = ops.reference.nvfp4_w4a4_linear(x.cpu(), p.cpu(), s.cpu(), g.cpu()) if M * N * K <= (1 << 31) else None
        err44 = None if ref44 is None else (ops.nvfp4_linear_w4a4(x, p, w_sf, s, g).float().cpu() - ref44).abs().max().item()
        packed = N * K // 2 + N * K // 16
        print(json.dumps({"shape": name, "M": M, "N": N, "K": K, "w4a16_us": round(t4, 2), "w4a4_us": round(t44, 2), "w4a4_quant_us": round(tq, 2), "mxfp8_w8a8_us": round(t8, 2),
                          "w4a4_gemm_nosplit_us": round(t_g1, 2), "w4a4_gemm_split_us": t_split,
                          "bf16_tcgen05_us": round(t16, 2), "cublas_bf16_us": round(tlib, 2),
                          "w4a4_packed_weight_gbs": round(packed / t44 / 1e3, 1),
                          "w4a4_speedup_vs_cublas_bf16": round(tlib / t44, 2),
                          "w4a16_speedup_vs_cublas_bf16": round(tlib / t4, 2),
                          "w4a16_max_abs_err_vs_dequantised": err, "w4a4_max_abs_err_vs_fp32_oracle": err44}))


def stamps_main(a):
    """Phase timeline of the stream-K kernel (in-kernel %globaltimer stamps, no profiler) for one config."""
    import statistics

    from vllm_suffix_hybrid_b200 import ops
    from vllm_suffix_hybrid_b200.ops.gemm import _sk_buffers

    kind, sw, bn, sp, cl = a.config.split(",")
    bn, nsub, cl = int(bn), int(sp), int(cl)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for name, M, N, K in SHAPES:
        if a.only and name not in a.only.split(","):
            continue
        x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.02
        y = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        nt = bn * nsub
        tiles = -(-N // 256) * -(-M // nt)
        ws, cnt = _sk_buffers(x.device, cl * 4 * nt * 128, 2 * tiles)
        st = torch.zeros(2 * cl, 64, dtype=torch.int64, device="cuda")
        for _ in range(3):
            flush.zero_()
            ops.native().gemm_bf16_sk(y, x, w, bn, nsub, cl, ws, cnt, None, st)
        torch.cuda.synchronize()
        t = st.cpu()
        t0 = int(t[:, 0].min())
        rel = lambda v: (int(v) - t0) / 1e3  # noqa: E731
        ends = [rel(t[i, 6]) for i in range(t.shape[0]) if t[i, 6] > 0]
        lead = [i for i in range(0, t.shape[0], 2)]
        summary = {
            "shape": name, "config": a.config, "tiles": tiles,
            "cta_end_us": {"min": round(min(ends), 2), "median": round(statistics.median(ends), 2), "max": round(max(ends), 2)},
            "dep_wait_done_us_median": round(statistics.median(rel(t[i, 2]) for i in range(t.shape[0])), 2),
            "producer_wait_free_stage_us_median": round(statistics.median(int(t[i, 3]) for i in range(t.shape[0])) / 1e3, 2),
            "mma_wait_loaded_stage_us_median": round(statistics.median(int(t[i, 4]) for i in lead) / 1e3, 2),
            "mma_wait_free_accumulator_us_median": round(statistics.median(int(t[i, 5]) for i in lead) / 1e3, 2),
            "segments_cta0": [[round(rel(t[0, 8 + 4 * j + q]), 2) if t[0, 8 + 4 * j + q] > 0 else None for q in range(4)]
                              for j in range(8) if t[0, 8 + 4 * j] > 0],
        }
        # the three CTAs that end last, with their segment timelines
        slow = sorted((i for i in range(t.shape[0]) if t[i, 6] > 0), key=lambda i: -int(t[i, 6]))[:3]
        summary["slowest"] = [{"cta": i, "end": round(rel(t[i, 6]), 2), "start": round(rel(t[i, 0]), 2),
                               "segments": [[round(rel(t[i, 8 + 4 * j + q]), 2) if t[i, 8 + 4 * j + q] > 0 else None
                                             for q in range(4)] for j in range(8) if (t[i, 8 + 4 * j:12 + 4 * j] > 0).any()],
                               "fixup_end": round(rel(t[i, 7]), 2) if t[i, 7] > 0 else None,
                               "fixup_us": round(int(t[i, 40]) / 1e3, 2), "fixup_store_us": round(int(t[i, 41]) / 1e3, 2),
                               "fixup_parts": int(t[i, 42])}
                              for i in slow]
        fx = [i for i in range(t.shape[0]) if t[i, 42] > 0]
        if fx:
            summary["fixups"] = {"ctas": len(fx), "parts_median": statistics.median(int(t[i, 42]) for i in fx),
                                 "us_median": round(statistics.median(int(t[i, 40]) for i in fx) / 1e3, 2),
                                 "us_max": round(max(int(t[i, 40]) for i in fx) / 1e3, 2),
                                 "store_us_median": round(statistics.median(int(t[i, 41]) for i in fx) / 1e3, 2)}
        print(json.dumps(summary), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--only", default="", help="comma-separated shape names")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--sweep", action="store_true", help="time every kernel configuration per shape")
    ap.add_argument("--once", action="store_true",
                    help="no timing: two eager launches of ours then cuBLAS per shape (for ncu captures)")
    ap.add_argument("--lib-only", action="store_true", help="with --once: launch only cuBLAS (profiling the library)")
    ap.add_argument("--stamps", action="store_true",
                    help="with --config sk,...: print the stream-K kernel's in-kernel phase timeline")
    ap.add_argument("--config", default="", help="force kind,swap,bn,splits,clusters (e.g. sk,1,192,2,74 or pair,0,256,1,0)")
    ap.add_argument("--w4a4", action="store_true", help="with --nvfp4 --once: launch the W4A4 kernel")
    ap.add_argument("--mxfp8", action="store_true", help="with --nvfp4 --once: launch the MXFP8 W8A8 kernel")
    ap.add_argument("--nvfp4", action="store_true",
                    help="NVFP4-weight (W4A16) kernel vs the bf16 paths on decode shapes (packed-weight GB/s)")
    a = ap.parse_args()
    if a.nvfp4:
        return nvfp4_main(a)
    if a.stamps:
        return stamps_main(a)
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
        if a.sweep:
            sweep(name, x, w, y, flush, a.iters)
        ours = lambda: tcgen05_linear(x, w, y)
        if a.config:
            from vllm_suffix_hybrid_b200.ops.gemm import Cfg, _runner

            kind, sw, bn, sp, cl = a.config.split(",")
            ours = _runner(Cfg(kind, bool(int(sw)), int(bn), int(sp), int(cl)), x, w, y)
        if a.once:
            for _ in range(2):
                flush.zero_()
                if not a.lib_only:
                    ours()
                flush.zero_()
                torch.matmul(x, w.t(), out=y)
            torch.cuda.synchronize()
            print(json.dumps({"once": name}))
            continue
        t_ours = time_fn(ours, flush, a.iters)
        t_lib = float("nan") if a.no_cublas else time_fn(lambda: torch.matmul(x, w.t(), out=y), flush, a.iters)
        ref = (x.float() @ w.float().t())
        tcgen05_linear(x, w, y)
        err = (y.float() - ref).abs().max().item()
        flops = 2.0 * M * N * K
        wbytes = N * K * 2
        r = {"shape": name, "M": M, "N": N, "K": K, "plan": plan(M, N, K, x, w, y)._asdict(), "tcgen05_us": round(t_ours, 2),
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
