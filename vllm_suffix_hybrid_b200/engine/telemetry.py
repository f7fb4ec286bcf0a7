"""Engine telemetry: periodic JSON stats lines and a JSONL stats file.

Same knobs as the reference's proposer telemetry (reference:
suffix_hybrid/hybrid_proposer.py:22-55):
  SUFFIX_HYBRID_LOG_INTERVAL    log a JSON stats line every N decode steps (0 = off)
  SUFFIX_HYBRID_STATS_FILE      append a JSONL record every
  SUFFIX_HYBRID_STATS_INTERVAL  N decode steps (default 100)
A record holds the proposer's native counters plus the engine's step,
accept-length and timing aggregates since the previous record.
"""
from __future__ import annotations

import json
import logging
import os
import time

logger = logging.getLogger("suffix_hybrid")


class Telemetry:
    def __init__(self, log_interval: int = 0, stats_file: str = "", stats_interval: int = 100):
        self.log_interval = max(0, log_interval)
        self.stats_file = stats_file
        self.stats_interval = max(1, stats_interval)
        self.steps = 0
        self._window = [0, 0, 0, 0.0, 0.0, 0.0]  # steps, rows, emitted, device_ms, host_ms, proposer_us

    @classmethod
    def from_env(cls) -> "Telemetry":
        def num(name, default):
            try:
                return int(os.environ.get(name, default))
            except ValueError:
                return default

        return cls(num("SUFFIX_HYBRID_LOG_INTERVAL", 0), os.environ.get("SUFFIX_HYBRID_STATS_FILE", "").strip(),
                   num("SUFFIX_HYBRID_STATS_INTERVAL", 100))

    @property
    def enabled(self) -> bool:
        return bool(self.log_interval or self.stats_file)

    def record(self, engine, step) -> None:
        self.steps += 1
        if not self.enabled:
            return
        w = self._window
        w[0] += 1
        w[1] += step.num_reqs
        w[2] += step.emitted
        w[3] += step.device_ms
        w[4] += step.host_ms
        w[5] += step.proposer_us
        log_due = self.log_interval and self.steps % self.log_interval == 0
        file_due = self.stats_file and self.steps % self.stats_interval == 0
        if not (log_due or file_due):
            return
        rec = {"ts": time.time(), "step": self.steps, "method": engine.cfg.spec.method, "k": engine.k,
               "window_steps": w[0], "mean_accept_len": w[2] / w[1] if w[1] else 0.0,
               "device_ms_per_step": w[3] / w[0], "host_ms_per_step": w[4] / w[0],
               "proposer_us_per_step": w[5] / w[0], "running": len(engine.running), "waiting": len(engine.waiting),
               "proposer": engine.proposer_stats()}
        line = json.dumps(rec, sort_keys=True, default=float)
        if log_due:
            logger.info("suffix_hybrid %s", line)
        if file_due:
            try:
                with open(self.stats_file, "a", encoding="utf-8") as fh:
                    fh.write(line + "\n")
            except OSError:
                logger.exception("suffix_hybrid cannot write telemetry")
        self._window = [0, 0, 0, 0.0, 0.0, 0.0]
