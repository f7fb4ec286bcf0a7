"""Proposer hot-path scaling benchmark (mixer + engine per decode step).

Same workload shape as the reference's harness (reference:
bench/scale_bench.py:20-95): `rows` requests with `ctx_len` tokens of
history built from a repeated 256-token block plus a distinct 8-token tail
per row; the mixer is measured with a cold and a warm corpus (64 sequences)
and the engine with suffix + n-gram.  Reports best and mean microseconds per
step.  Run: python -m vllm_suffix_hybrid_b200.bench.scale_bench
"""
import argparse
import json
import time

import numpy as np

from vllm_suffix_hybrid_b200._native import Engine, HybridMixer


def make_batch(rows, ctx_len, k, vocab=50_000, seed=7):
    rng = np.random.default_rng(seed)
    block = rng.integers(1000, vocab, size=256, dtype=np.int64)
    width = ctx_len + k + 8
    tokens = np.zeros((rows, width), dtype=np.int64)
    for i in range(rows):
        tokens[i, :] = np.tile(block, (width + 255) // 256)[:width]
        tokens[i, ctx_len - 8:ctx_len] = rng.integers(1000, vocab, size=8)
    counts = np.full(rows, ctx_len, dtype=np.int64)
    ids = [f"req-{i}" for i in range(rows)]
    drafts = [[int(tokens[i, ctx_len + j]) for j in range(k)] for i in range(rows)]
    return ids, counts, tokens, drafts


def bench_mixer(rows, ctx_len, k, steps, warm):
    mixer = HybridMixer(k, ctx_len + 4096)
    if warm:
        for s in range(64):
            mixer.suffix_cache.add_sequence(np.tile(np.arange(256, dtype=np.int64) + 1000 * s, ctx_len // 256))
    ids, counts, tokens, drafts = make_batch(rows, ctx_len, k)
    accepted = [k] * rows
    mixer.mix_numpy(ids, counts, tokens, drafts, None)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter_ns()
        mixer.mix_numpy(ids, counts, tokens, drafts, accepted)
        times.append(time.perf_counter_ns() - t0)
    return min(times) / 1e3, sum(times) / len(times) / 1e3


def bench_engine(rows, ctx_len, k, steps):
    engine = Engine(k, ctx_len + 4096)
    ids, counts, tokens, drafts = make_batch(rows, ctx_len, k)
    sampled = [[int(tokens[i, ctx_len])] for i in range(rows)]
    engine.propose(sampled, counts, tokens)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter_ns()
        engine.propose(sampled, counts, tokens)
        times.append(time.perf_counter_ns() - t0)
    return min(times) / 1e3, sum(times) / len(times) / 1e3


def run(rows=16, ctx_len=8192, k=4, steps=40):
    out = {}
    for label, fn in (
        ("mixer_cold", lambda: bench_mixer(rows, ctx_len, k, steps, False)),
        ("mixer_warm", lambda: bench_mixer(rows, ctx_len, k, steps, True)),
        ("engine", lambda: bench_engine(rows, ctx_len, k, steps)),
    ):
        best, mean = fn()
        out[label] = {"best_us": round(best, 3), "mean_us": round(mean, 3)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, default=16)
    ap.add_argument("--len", dest="ctx_len", type=int, default=8192)
    ap.add_argument("--k", type=int, default=4)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    res = run(a.rows, a.ctx_len, a.k, a.steps)
    if a.json:
        print(json.dumps(res))
        return
    print(f"rows={a.rows} ctx_len={a.ctx_len} k={a.k} steps={a.steps}")
    print(f"{'path':<14}{'best_us':>10}{'mean_us':>10}")
    for label, r in res.items():
        print(f"{label:<14}{r['best_us']:>10.3f}{r['mean_us']:>10.3f}")


if __name__ == "__main__":
    main()
