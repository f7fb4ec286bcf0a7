"""Headline benchmark: decode output tokens/s per box with k=5 hybrid speculation.

Workload (benchmark config 1): Llama-3-8B-shaped decoder, bf16 random init
N(0, 0.02), a 1-layer EAGLE-style draft head of the same width, k = 5 greedy
hybrid speculation (native drafts mixed with the suffix corpus by the native
mixer), 64 concurrent requests with synthetic 2048-token prompts (config-0
span-reuse structure, vocab 128256), up to 512 output tokens each.  On N GPUs
the model runs tensor-parallel over N ranks (one process per GPU, NCCL).

Timed region: K decode steps after W warm-up steps, bracketed by a barrier
and a device synchronize.  Before the warm-up the generation is advanced
(untimed) so that the W + K steps are centred on the middle of the
max-new-token generation: the timed steps see the mean context length of the
run, not the shortest one right after prefill.  `value` is output tokens / summed device time of
the steps (CUDA events from the H2D of a step's inputs to the D2H of its
results, max over ranks).  `e2e` is the same tokens over the wall clock of
the K `LLMEngine.step()` calls, which include the host proposer, the H2D of
each step's inputs from pinned memory and the D2H of its results.  The
per-step working set (16 GB of weights + the KV cache) is far larger than the
126 MB L2, so no L2 flush is inserted between steps.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""
import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


# Per-config workload: requests, prompt and output lengths, layout.
CONFIG_DEFAULTS = {
    "llama3-8b": dict(batch=64, prompt_len=2048, max_new=512, layout="tp", synthetic_prefill=False),
    "qwen3-next": dict(batch=32, prompt_len=8192, max_new=1024, layout="dp-ep", synthetic_prefill=True),
    "deepseek-v3.2": dict(batch=32, prompt_len=32768, max_new=1024, layout="dp-ep", synthetic_prefill=True),
    "kimi-k2": dict(batch=64, prompt_len=131072, max_new=1024, layout="dp-ep", synthetic_prefill=True,
                    streams=dict(p_copy=0.6, corpus_n=256), env={"SUFFIX_HYBRID_NGRAM_WINDOW": "8192"}),
}


def reference_arm(args):
    why = ("reference build backend unavailable offline: the reference is a maturin (Rust/PyO3) package and "
           "neither maturin nor cargo is installed; its native module suffix_hybrid._native cannot be built, "
           "and the plugin needs vLLM at its pinned revision")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": why}))


def trace_steps(eng, path, rank, barrier):
    """Per-kernel device time of 2 decode steps (torch.profiler / CUPTI), summed by kernel name."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile

    barrier()
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(2):
            eng.step()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    spans = []
    for ev in prof.events():
        if ev.device_type is not None and str(ev.device_type).endswith("CUDA") and ev.device_time_total > 0:
            name = ev.name
            agg[name][0] += 1
            agg[name][1] += ev.device_time_total
            spans.append((ev.time_range.start, ev.time_range.end))
    total = sum(v[1] for v in agg.values())
    busy, end = 0.0, None
    for a, b in sorted(spans):
        if end is None or a > end:
            busy += b - a
            end = b
        elif b > end:
            busy += b - end
            end = b
    wall = (max(b for _, b in spans) - min(a for a, _ in spans)) if spans else 0.0
    with open(f"{path}_rank{rank}.txt", "w") as fh:
        fh.write(f"# 2 decode steps; kernel time {total:.1f} us; device busy {busy:.1f} us of {wall:.1f} us span\n")
        for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
            fh.write(f"{t:10.1f} us {n:6d}  {100 * t / max(total, 1e-9):5.1f}%  {name[:150]}\n")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=32)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="llama3-8b")
    ap.add_argument("--method", default="hybrid")
    ap.add_argument("--split", default="legacy")
    ap.add_argument("--batch", type=int, default=0, help="global requests (default: the config's)")
    ap.add_argument("--prompt-len", type=int, default=0, help="prompt tokens (default: the config's)")
    ap.add_argument("--max-new", type=int, default=0, help="output tokens per request (default: the config's)")
    ap.add_argument("--layout", default="", choices=["", "tp", "dp-ep"],
                    help="tp: tensor parallel over the N GPUs; dp-ep: data-parallel attention (each rank serves "
                         "its own requests) with the MoE experts split over the N ranks (default: the config's)")
    ap.add_argument("--synthetic-prefill", default="", choices=["", "0", "1"],
                    help="1: admit the prompts with a randomly filled KV cache instead of running the prefill "
                         "forward (long-context decode benches; default: on for the 32k/128k configs)")
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--timed-from", type=int, default=-1,
                    help="generated tokens per request before the warm-up steps start (default: the timed window "
                         "is centred on the middle of the max-new-token generation, the mean context length)")
    ap.add_argument("--adaptive-width", action="store_true",
                    help="verify only as wide as the longest real draft (off for the headline: every step "
                         "verifies k + 1 tokens per row)")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                    help="TP collectives: own NVLink kernels (fused) or the NCCL baseline")
    ap.add_argument("--layers", type=int, default=0, help="debug only: override layer count (invalid for bench)")
    ap.add_argument("--profile", action="store_true",
                    help="profile one eager decode step between cudaProfilerStart/Stop (for ncu) and exit")
    ap.add_argument("--dump-tokens", type=int, default=0, help="print the first N generated tokens of row 0")
    ap.add_argument("--trace", default="",
                    help="after the timed steps, run 2 untimed steps under torch.profiler and write a per-kernel "
                         "device-time summary per rank to <trace>_rank<R>.txt")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_arm(args)
        return
    import faulthandler

    t_start = time.perf_counter()

    def progress(msg):  # stderr breadcrumbs: a run that is killed still shows how far it got
        print(f"[bench +{time.perf_counter() - t_start:7.1f}s rank {os.environ.get('RANK', '0')}] {msg}",
              file=sys.stderr, flush=True)

    if os.environ.get("SH_BENCH_STACKS_AFTER_S"):  # dump every thread's stack if still running after N s
        faulthandler.dump_traceback_later(float(os.environ["SH_BENCH_STACKS_AFTER_S"]), exit=False)

    import numpy as np
    import torch
    import torch.distributed as dist

    from vllm_suffix_hybrid_b200 import ops
    from vllm_suffix_hybrid_b200.bench.synthetic import make_streams
    from vllm_suffix_hybrid_b200.engine.config import PRESETS, CacheConfig, EngineConfig, ParallelConfig, SpecConfig
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine
    from vllm_suffix_hybrid_b200.parallel import state as pstate
    from vllm_suffix_hybrid_b200.utils.clocks import ClockSampler

    d = CONFIG_DEFAULTS[args.config]
    args.batch = args.batch or d["batch"]
    args.prompt_len = args.prompt_len or d["prompt_len"]
    args.max_new = args.max_new or d["max_new"]
    layout = args.layout or d["layout"]
    synthetic = (args.synthetic_prefill or ("1" if d["synthetic_prefill"] else "0")) == "1"
    for key, val in d.get("env", {}).items():
        os.environ.setdefault(key, val)
    n = args.gpus
    if layout == "dp-ep" and n > 1:
        st = pstate.init(ep=n, dp=n)
    else:
        st = pstate.init(tp=n)
    rank, world = st.rank, st.world
    assert world == args.gpus, f"--gpus {args.gpus} but WORLD_SIZE {world}"
    if layout == "dp-ep" and args.batch % max(world, 1):
        raise SystemExit(f"--batch {args.batch} must split evenly over {world} data-parallel ranks")
    local_batch = args.batch // world if layout == "dp-ep" else args.batch
    mcfg = PRESETS[args.config]()
    if args.layers:
        mcfg.layers = args.layers
    par = (ParallelConfig(ep=n, dp=n, comm=args.comm) if layout == "dp-ep" and n > 1
           else ParallelConfig(tp=n, comm=args.comm))
    cfg = EngineConfig(model=mcfg, spec=SpecConfig(method=args.method, k=args.k, split=args.split,
                                                   adaptive_width=args.adaptive_width),
                       parallel=par,
                       cache=CacheConfig(max_model_len=args.prompt_len + args.max_new + 4 * args.k + 64),
                       max_num_seqs=local_batch, device="cuda", cuda_graphs=not args.no_graphs)
    if args.split == "diverge":
        os.environ["SUFFIX_HYBRID_SPLIT"] = "diverge"
    progress("building the engine")
    eng = LLMEngine(cfg)
    progress("engine ready; prefill")
    prompts = make_streams(args.batch, args.prompt_len, mcfg.vocab, seed=1234, **d.get("streams", {}))
    mine = prompts[rank::world] if layout == "dp-ep" else prompts
    t_pf = time.perf_counter()
    if synthetic:
        eng.admit_prefilled(mine, args.max_new, seed=1234 + rank)
    else:
        for p in mine:
            eng.add_request(p, args.max_new)
        while eng.waiting:
            eng.step()
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t_pf

    def barrier():
        if world > 1:
            dist.barrier(group=st.cpu_group)

    # Untimed decode up to the start of the window: attention cost grows with the context, so the timed
    # steps sit around the middle of the generation instead of right after prefill.  Every rank runs the
    # same steps (the engine state is replicated), so the loop ends on the same step everywhere.
    start_at = args.timed_from if args.timed_from >= 0 else max(0, args.max_new // 2 - (args.warmup + args.steps) // 2)
    progress(f"prefill done in {prefill_s:.1f}s; advancing to {start_at} generated tokens")
    def below_start() -> bool:
        """Whether any request (on any rank, in the data-parallel layout) is short of the window start."""
        mine = bool(eng.running) and min(len(r.output) for r in eng.running) < start_at
        if layout == "dp-ep" and world > 1:  # ranks step in lockstep: agree on the loop's end
            flag = torch.tensor([1 if mine else 0], dtype=torch.int32)
            dist.all_reduce(flag, group=st.cpu_group)
            return int(flag.item()) > 0
        return mine

    advanced = 0
    while below_start():
        eng.step()
        advanced += 1
        if advanced % 50 == 0:
            progress(f"advanced {advanced} steps")
    progress(f"advanced {advanced} steps; warm-up")
    for _ in range(args.warmup):
        eng.step()
    progress("timed steps")
    if args.profile:
        eng.runner.use_graphs = False
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        eng.step()
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profiled_step": True, "num_reqs": len(eng.running)}))
        return
    # Kernel launches of this framework per decode step (one eager step, counted).
    n_launch_step = 0
    if cfg.cuda_graphs:
        r = eng.runner
        ctr = ops.count_launches(True)
        nb, wd = max(r.graphs, key=lambda kw: (kw[0] == len(eng.running), kw[1]))
        r._decode_body(nb, wd)
        ops.count_launches(False)
        n_launch_step = ctr.count
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(gpus=list(range(world)))
    if rank == 0:
        clocks.start()
    torch.cuda.synchronize()
    barrier()
    first = len(eng.stats)
    ctx0 = min(len(r.prompt) + len(r.output) for r in eng.running) if eng.running else 0
    t0 = time.perf_counter()
    dev_ms = 0.0
    h2d = d2h = 0
    width_sum = 0
    for _ in range(args.steps):
        s = eng.step()
        assert s.kind == "decode", s
        dev_ms += eng.runner.last_device_ms
        width_sum += eng.runner.last_width
        h2d += eng.runner.h2d_bytes
        d2h += eng.runner.d2h_bytes
    torch.cuda.synchronize()
    barrier()
    wall = time.perf_counter() - t0
    clk = clocks.stop() if rank == 0 else {}
    steps = eng.stats[first:]
    tokens = sum(s.emitted for s in steps)
    rows = sum(s.num_reqs for s in steps)
    prop_us = sum(s.proposer_us for s in steps) / len(steps)
    t = torch.tensor([dev_ms, wall], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=st.group)
    dev_ms, wall = float(t[0]), float(t[1])
    if layout == "dp-ep" and world > 1:  # every rank emits for its own requests: the box's output is the sum
        c = torch.tensor([tokens, rows], dtype=torch.float64, device="cuda")
        dist.all_reduce(c, group=st.group)
        tokens, rows = int(c[0]), int(c[1])
    from vllm_suffix_hybrid_b200.ops import gemm as _gemm

    gemm_choices = _gemm.choice_summary()
    if rank == 0:
        value = tokens / (dev_ms / 1e3)
        e2e = tokens / wall
        out = {
            "metric": "decode out tok/s/box w/ k=5 hybrid spec (max over ranks); mean accept len; us/step",
            "value": round(value, 1),
            "unit": "tok/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dev_ms / args.steps, 3),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": (f"synthetic (span-reuse token streams, vocab {mcfg.vocab}); random-init weights "
                     f"({mcfg.weight_format})" + ("; prompts admitted with a random-filled KV cache (prefill "
                                                  "forward skipped, every decode step complete)" if synthetic else "")),
            "config": {"model": "llama3-8b-shape" if args.config == "llama3-8b" else f"{args.config}-shape",
                       "global_batch": args.batch, "seq_len": args.prompt_len, "max_new_tokens": args.max_new,
                       "k": args.k, "method": args.method, "split": args.split,
                       "parallelism": (f"dp{world}-ep{world}" if layout == "dp-ep" and world > 1 else f"tp{world}"),
                       "comm": args.comm if world > 1 else "none",
                       "l2": "working set (weights + KV) >> 126 MB L2; no flush",
                       "layers": mcfg.layers, "weights": mcfg.weight_format, "kv_cache": mcfg.kv_format},
            "mean_accept_len": round(tokens / rows, 4),
            "mean_verify_width": round(width_sum / args.steps, 3),
            "adaptive_width": bool(args.adaptive_width),
            "timed_window": {"untimed_steps_before_warmup": advanced, "min_context_at_first_timed_step": ctx0},
            "proposer_us_per_step": round(prop_us, 2),
            "prefill_s": round(prefill_s, 2),
            "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d // args.steps,
                    "d2h_bytes_per_step": d2h // args.steps, "api": "LLMEngine.step"},
            "gpu_launches": n_launch_step * args.steps,
            "clocks": clk,
            "gemm_choices": gemm_choices,
            "impl": "ours",
        }
        if args.layers:
            out["invalid"] = "layer count overridden (debug run)"
        if args.dump_tokens:
            r0 = eng.running[0]
            out["sample_tokens"] = r0.output[: args.dump_tokens]
        print(json.dumps(out))
    if args.trace:
        try:
            trace_steps(eng, args.trace, rank, barrier)
        except Exception as e:  # diagnostics only; never fail the benchmark
            print(f"trace failed on rank {rank}: {e!r}", file=sys.stderr)
    if world > 1:
        eng.runner.graphs.clear()
        torch.cuda.synchronize()
        pstate.shutdown()


if __name__ == "__main__":
    main()
