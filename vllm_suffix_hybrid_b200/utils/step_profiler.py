"""Step profiler: torch.profiler windows over engine steps, bucketed by batch size.

Knobs (the reference's step profiler windows work the same way, reference:
suffix_hybrid/step_profiler.py:126,370,682):
  SUFFIX_HYBRID_STEP_PROFILE=<dir>       enable; traces and summaries go to <dir>
  SUFFIX_HYBRID_STEP_PROFILE_SKIP=<n>    decode steps to skip first (default 20)
  SUFFIX_HYBRID_STEP_PROFILE_STEPS=<n>   steps per window (default 5)
  SUFFIX_HYBRID_STEP_PROFILE_BUCKETS=8,32,64   one window per running-batch bucket (batch <= bucket)
Each window writes a Chrome trace (<dir>/step_b<bucket>_r<rank>.json) and a per-kernel device-time
summary (<dir>/step_b<bucket>_r<rank>.txt: total, count, share, name).
"""
from __future__ import annotations

import collections
import os
from typing import Optional


class StepProfiler:
    def __init__(self, out_dir: str, skip: int = 20, steps: int = 5, buckets=(8, 32, 64), rank: int = 0):
        self.dir, self.skip, self.steps, self.rank = out_dir, skip, steps, rank
        self.buckets = sorted(buckets)
        self.done = set()
        self.seen = 0
        self.prof = None
        self.bucket: Optional[int] = None
        self.count = 0
        os.makedirs(out_dir, exist_ok=True)

    @classmethod
    def from_env(cls, rank: int = 0) -> Optional["StepProfiler"]:
        d = os.environ.get("SUFFIX_HYBRID_STEP_PROFILE", "").strip()
        if not d:
            return None
        b = os.environ.get("SUFFIX_HYBRID_STEP_PROFILE_BUCKETS", "8,32,64")
        return cls(d, int(os.environ.get("SUFFIX_HYBRID_STEP_PROFILE_SKIP", "20")),
                   int(os.environ.get("SUFFIX_HYBRID_STEP_PROFILE_STEPS", "5")),
                   [int(x) for x in b.split(",") if x.strip()], rank)

    def _bucket(self, batch: int) -> Optional[int]:
        return next((x for x in self.buckets if batch <= x), None)

    def before(self, kind: str, batch: int) -> None:
        if kind != "decode" or self.prof is not None:
            return
        self.seen += 1
        b = self._bucket(batch)
        if self.seen <= self.skip or b is None or b in self.done:
            return
        import torch
        from torch.profiler import ProfilerActivity, profile

        acts = [ProfilerActivity.CPU] + ([ProfilerActivity.CUDA] if torch.cuda.is_available() else [])
        self.prof = profile(activities=acts)
        self.prof.__enter__()
        self.bucket, self.count = b, 0

    def after(self) -> None:
        if self.prof is None:
            return
        self.count += 1
        if self.count < self.steps:
            return
        import torch

        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.prof.__exit__(None, None, None)
        base = os.path.join(self.dir, f"step_b{self.bucket}_r{self.rank}")
        try:
            self.prof.export_chrome_trace(base + ".json")
        except Exception:
            pass
        agg = collections.defaultdict(lambda: [0, 0.0])
        for ev in self.prof.events():
            if ev.device_type is not None and str(ev.device_type).endswith("CUDA") and ev.device_time_total > 0:
                agg[ev.name][0] += 1
                agg[ev.name][1] += ev.device_time_total
        total = sum(v[1] for v in agg.values()) or 1.0
        with open(base + ".txt", "w") as fh:
            fh.write(f"# {self.count} decode steps, batch bucket <= {self.bucket}; device kernel time {total:.1f} us\n")
            for name, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
                fh.write(f"{t:10.1f} us {n:6d} {100 * t / total:5.1f}%  {name[:160]}\n")
        self.done.add(self.bucket)
        self.prof = None
