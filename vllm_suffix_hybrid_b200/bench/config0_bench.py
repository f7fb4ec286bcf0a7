"""Config 0: the proposer loop on the CPU with a toy target that verifies.

Workload (benchmark config 0): 16 rows of 8192-token histories built by the
span-reuse generator (``bench.synthetic.make_streams``: segments that copy a
U[16, 256] span from earlier in the row or from a shared 64-sequence corpus
of 4096 Zipf(1.1) tokens with p = 0.4, else 32-128 i.i.d. Zipf tokens),
vocab 32000.  Target: the 2-layer, 256-dim, 4-head fp32 random-init decoder;
native drafter: its 1-layer MTP head; k = 5.  The whole engine runs on the
CPU: prefill of the 16 histories, then decode steps in which the proposer
(hybrid mixer over the suffix corpus + the MTP head's drafts, or the
weight-free suffix + n-gram Engine) proposes, the toy target verifies the
k + 1 window greedily, and every row appends its accepted tokens
(incremental histories: the proposers only read each row's delta).

Reports per-step proposer microseconds (mixer for ``hybrid``, engine for
``ngram``), the C++ core's share where the proposer exposes it, and the mean
accepted length per row-step.  The reference publishes 4.7 us (mixer) and
118 us (engine) per step at 16 rows x 8k (reference: README.md:97-100, its
harness bench/scale_bench.py:41-95 times a static batch; this bench runs
the verify loop).

Run: python -m vllm_suffix_hybrid_b200.bench.config0_bench [--steps 64] [--json]
"""
from __future__ import annotations

import argparse
import json
import time

import numpy as np


def run(method: str, rows: int, ctx: int, steps: int, k: int, seed: int, threads: int) -> dict:
    import torch

    from vllm_suffix_hybrid_b200.bench.synthetic import make_streams
    from vllm_suffix_hybrid_b200.engine.config import CacheConfig, EngineConfig, SpecConfig, toy_config
    from vllm_suffix_hybrid_b200.engine.llm import LLMEngine

    if threads:
        torch.set_num_threads(threads)
    m = toy_config()
    gen = steps * (k + 1) + 8
    cfg = EngineConfig(model=m, spec=SpecConfig(method=method, k=k),
                       cache=CacheConfig(max_model_len=ctx + gen + 4 * k + 64), max_num_seqs=rows, device="cpu",
                       cuda_graphs=False, max_prefill_tokens=2 * ctx)
    eng = LLMEngine(cfg)
    streams = make_streams(rows, ctx, m.vocab, seed=seed)
    # The shared corpus the streams copy from is what a serving corpus would have seen: the first half of
    # the rows' histories are given to the suffix corpus as finished requests (cross-request reuse).
    eng.warm_start([s[: ctx // 2] for s in streams])
    for s in streams:
        eng.add_request(s, gen)
    t0 = time.perf_counter()
    while eng.waiting:
        eng.step()
    prefill_s = time.perf_counter() - t0
    first = len(eng.stats)
    t0 = time.perf_counter()
    for _ in range(steps):
        if not eng.running:
            break
        eng.step()
    wall = time.perf_counter() - t0
    dec = [s for s in eng.stats[first:] if s.kind == "decode"]
    rows_steps = sum(s.num_reqs for s in dec)
    prop = [s.proposer_us for s in dec]
    out = {"method": method, "rows": rows, "ctx": ctx, "k": k, "decode_steps": len(dec),
           "proposer_us_mean": round(float(np.mean(prop)), 2) if prop else None,
           "proposer_us_best": round(float(np.min(prop)), 2) if prop else None,
           "proposer_us_median": round(float(np.median(prop)), 2) if prop else None,
           "mean_accept_len": round(sum(s.emitted for s in dec) / max(rows_steps, 1), 4),
           "prefill_s": round(prefill_s, 2), "decode_wall_ms_per_step": round(1e3 * wall / max(len(dec), 1), 2)}
    st = eng.proposer_stats() if hasattr(eng, "proposer_stats") else {}
    if isinstance(st, dict):
        for key in ("native_time_ns", "total_proposer_time_ns", "calls", "suffix_proposals", "ngram_proposals"):
            if key in st:
                out["proposer_" + key] = st[key]
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=16)
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--threads", type=int, default=0)
    ap.add_argument("--methods", default="hybrid,ngram")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    res = [run(mth, a.rows, a.ctx, a.steps, a.k, a.seed, a.threads) for mth in a.methods.split(",")]
    line = {"metric": "config-0 proposer us/step (mixer: hybrid, engine: ngram) and mean accept len",
            "data": "synthetic span-reuse streams (make_streams, vocab 32000); toy fp32 target + 1-layer MTP head, "
                    "random init", "device": "cpu", "results": res,
            "reference_published_us": {"mixer": 4.7, "engine": 118.0}}
    print(json.dumps(line) if a.json else json.dumps(line, indent=1))


if __name__ == "__main__":
    main()
