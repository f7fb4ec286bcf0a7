"""Acceptance simulator for the speculative proposers (CPU only).

Tokens emitted per verify step on scripted workloads whose greedy continuation is known.  The package's
native HybridMixer is driven the way ``LLMEngine`` drives it: every step it gets each row's verified
context, the draft head's proposal and the row's accepted length from the previous step, and rows that
leave the batch go into the shared suffix corpus.  The target is replaced by the known continuation, and
the draft head by a model of one:

* a draft position is right with a probability that falls with its depth in the window, higher where the
  true token repeats text seen earlier in the row;
* once a position is wrong, every later position is wrong too (it was conditioned on a wrong prefix);
* greedy verification accepts the longest prefix that matches the continuation, plus the bonus token.

Workloads (the categories the reference's simulator measures, reference: bench/spec_sim.py:1-25):

* ``fresh``     new text with a few short self-repeats;
* ``templated`` a handful of requests that recur, so their continuations recur word for word;
* ``echo``      the continuation repeats the prompt with sparse edits;
* ``tools``     multi-turn sessions whose turns quote spans of the growing history.

Arms: ``draft`` (the draft head alone), ``hybrid`` (mixer, legacy split), ``diverge`` (mixer, diverge
split).  Absolute numbers depend on the draft-head model; the gap between arms on the same seeded
workload is the measurement.

Run: python -m vllm_suffix_hybrid_b200.bench.spec_sim [--k 5] [--conc 1,8] [--requests 48] [--json]
"""
from __future__ import annotations

import argparse
import json
import os
import time
from typing import Dict, Iterator, List, Tuple

import numpy as np

VOCAB = 32000
GEN = 256
# draft head model: P(position t right | earlier ones right) = base * decay ** t
HEAD_FRESH = (0.78, 0.90)
HEAD_REPEAT = (0.94, 0.975)

Job = Tuple[List[int], List[int], List[bool]]  # prompt, continuation, "repeats earlier text" per token


def _words(rng: np.random.Generator, n: int) -> List[int]:
    """Skewed unigram draws, so short n-grams recur by chance as in real text."""
    return (rng.random(n) ** 2.5 * VOCAB).astype(np.int64).tolist()


def workload(name: str, n_req: int, seed: int = 0, gen: int = GEN) -> Iterator[Job]:
    rng = np.random.default_rng(seed)
    if name == "fresh":
        for _ in range(n_req):
            out: List[int] = []
            rep: List[bool] = []
            while len(out) < gen:
                if len(out) > 48 and rng.random() < 0.04:
                    L = int(rng.integers(6, 13))
                    s = int(rng.integers(0, len(out) - L))
                    out += out[s:s + L]
                    rep += [True] * L
                else:
                    out += _words(rng, 1)
                    rep.append(False)
            yield _words(rng, 48), out[:gen], rep[:gen]
    elif name == "templated":
        temps = [(_words(rng, 48), _words(rng, gen)) for _ in range(5)]
        for i in range(n_req):
            p, c = temps[i % len(temps)]
            yield list(p), list(c), [False] * gen
    elif name == "echo":
        for _ in range(n_req):
            passage = _words(rng, 180)
            src = (passage * 2)[:gen]
            edits = rng.random(gen) < 0.03
            noise = _words(rng, gen)
            out = [noise[i] if edits[i] else t for i, t in enumerate(src)]
            yield passage + _words(rng, 10), out, [True] * gen
    elif name == "tools":
        for _ in range(max(1, n_req // 5)):
            history = _words(rng, 360)
            for _turn in range(5):
                prompt = history + _words(rng, 90)  # the new tool output
                out, rep = [], []
                while len(out) < gen:
                    if rng.random() < 0.55:
                        L = int(rng.integers(12, 49))
                        s = int(rng.integers(0, max(1, len(prompt) - L)))
                        out += prompt[s:s + L]
                        rep += [True] * L
                    else:
                        L = int(rng.integers(4, 21))
                        out += _words(rng, L)
                        rep += [False] * L
                yield prompt, out[:gen], rep[:gen]
                history = prompt + out[:gen]
    else:
        raise ValueError(f"unknown workload {name!r}")


def head_draft(rng: np.random.Generator, truth: List[int], rep: List[bool], k: int) -> List[int]:
    """The draft head's k tokens for the next window (truth: the continuation from the window start)."""
    out, right = [], True
    for t in range(k):
        if t >= len(truth):
            out += _words(rng, 1)
            continue
        base, decay = HEAD_REPEAT if rep[t] else HEAD_FRESH
        if right and rng.random() < base * decay ** t:
            out.append(truth[t])
        else:
            right = False
            w = _words(rng, 1)[0]
            out.append(w if w != truth[t] else (w + 1) % VOCAB)
    return out


def simulate(name: str, arm: str, k: int = 5, conc: int = 8, n_req: int = 48, seed: int = 0) -> Dict:
    """Run one workload through one arm; returns emitted / accepted tokens per row step and host time."""
    from vllm_suffix_hybrid_b200 import _native

    saved = os.environ.get("SUFFIX_HYBRID_SPLIT")
    if arm == "diverge":
        os.environ["SUFFIX_HYBRID_SPLIT"] = "diverge"
    else:
        os.environ.pop("SUFFIX_HYBRID_SPLIT", None)
    try:
        mixer = None if arm == "draft" else _native.HybridMixer(k, 1 << 20)
    finally:
        if saved is None:
            os.environ.pop("SUFFIX_HYBRID_SPLIT", None)
        else:
            os.environ["SUFFIX_HYBRID_SPLIT"] = saved
    rng = np.random.default_rng(seed + 7)
    pending = list(workload(name, n_req, seed))
    live: Dict[str, dict] = {}
    n_id = 0
    row_steps = emitted = accepted = 0
    host_ns = calls = 0
    while pending or live:
        while pending and len(live) < conc:
            p, c, rep = pending.pop(0)
            # prefill emits the first continuation token
            live[f"q{n_id}"] = dict(ctx=p + c[:1], truth=c, rep=rep, pos=1, acc=-1)
            n_id += 1
        ids = list(live)
        heads = [head_draft(rng, live[r]["truth"][live[r]["pos"]:live[r]["pos"] + k],
                            live[r]["rep"][live[r]["pos"]:live[r]["pos"] + k], k) for r in ids]
        if mixer is None:
            drafts = heads
        else:
            t0 = time.perf_counter_ns()
            drafts = mixer.mix(ids, [live[r]["ctx"] for r in ids], heads, [live[r]["acc"] for r in ids])
            host_ns += time.perf_counter_ns() - t0
            calls += 1
        for r, d in zip(ids, drafts):
            s = live[r]
            truth, pos = s["truth"], s["pos"]
            a = 0
            while a < len(d) and pos + a < len(truth) and d[a] == truth[pos + a]:
                a += 1
            step = truth[pos:pos + a + 1]  # accepted drafts + the target's bonus token
            s["ctx"] = s["ctx"] + step
            s["pos"] = pos + len(step)
            s["acc"] = a
            row_steps += 1
            emitted += len(step)
            accepted += a
            if s["pos"] >= len(truth):
                del live[r]
    stats = {}
    if mixer is not None:
        mixer.mix([], [], [], [])  # the last departures enter the corpus
        st = mixer.get_stats()
        stats = {key: st[key] for key in ("native_accepted", "suffix_accepted", "suffix_proposed", "div_observed",
                                          "div_suffix_published", "self_hits") if key in st}
    return {"tokens_per_step": emitted / max(row_steps, 1), "accepted_per_step": accepted / max(row_steps, 1),
            "row_steps": row_steps, "host_us_per_call": host_ns / 1e3 / max(calls, 1), "stats": stats}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--k", type=int, default=5)
    ap.add_argument("--conc", default="1,8")
    ap.add_argument("--requests", type=int, default=48)
    ap.add_argument("--workloads", default="fresh,templated,echo,tools")
    ap.add_argument("--arms", default="draft,hybrid,diverge")
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    rows = []
    for name in a.workloads.split(","):
        for conc in (int(c) for c in a.conc.split(",")):
            for arm in a.arms.split(","):
                r = simulate(name, arm, a.k, conc, a.requests)
                rows.append({"workload": name, "conc": conc, "arm": arm, **r})
                if not a.json:
                    print(f"{name:10s} c={conc:<3d} {arm:8s} tok/step={r['tokens_per_step']:.3f} "
                          f"acc/step={r['accepted_per_step']:.3f} host={r['host_us_per_call']:.1f}us {r['stats']}")
    if a.json:
        print(json.dumps(rows))


if __name__ == "__main__":
    main()
