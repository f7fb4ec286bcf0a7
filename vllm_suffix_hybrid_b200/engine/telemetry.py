"""Telemetry: periodic JSON stats lines and an append-only JSONL stats file.

Knobs (the reference's proposer telemetry reads the same variables,
reference: suffix_hybrid/hybrid_proposer.py:22-55):
  SUFFIX_HYBRID_LOG_INTERVAL    log a JSON stats line every N events
  SUFFIX_HYBRID_STATS_FILE      append a JSONL record every
  SUFFIX_HYBRID_STATS_INTERVAL  N events (default 100)

Two producers share one sink:

* ``Telemetry`` -- the engine's decode steps.  A record holds the
  proposer's native counters plus the step, accept-length and timing
  aggregates since the previous record.  Logging is off unless
  SUFFIX_HYBRID_LOG_INTERVAL is set.
* ``CallTelemetry`` -- calls of a stand-alone proposer object (the
  custom-class ``HybridProposer``).  A record is the proposer's own
  ``get_stats()`` dictionary; logging defaults to every 100 calls.

Writing a record is timed too, and the time is charged to the proposer
(``record_total``), so the reported proposer time is what the caller saw.
"""
from __future__ import annotations

import json
import logging
import os
import time
from typing import Callable, Optional

logger = logging.getLogger("suffix_hybrid")


def _env_int(name: str, default: int) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class _Sink:
    """Where records go: the logger, the JSONL file, or both."""

    def __init__(self, log_interval: int, stats_file: str, stats_interval: int):
        self.log_interval = max(0, log_interval)
        self.stats_file = stats_file
        self.stats_interval = max(1, stats_interval)

    @property
    def enabled(self) -> bool:
        return bool(self.log_interval or self.stats_file)

    def due(self, count: int):
        """(log now, append to the file now) after the count-th event."""
        return (bool(self.log_interval) and count % self.log_interval == 0,
                bool(self.stats_file) and count % self.stats_interval == 0)

    def write(self, rec: dict, to_log: bool, to_file: bool) -> None:
        line = json.dumps(rec, sort_keys=True, default=float)
        if to_log:
            logger.info("suffix_hybrid %s", line)
        if to_file:
            try:
                with open(self.stats_file, "a", encoding="utf-8") as fh:
                    fh.write(line + "\n")
            except OSError:
                logger.exception("suffix_hybrid cannot write telemetry")


class Telemetry(_Sink):
    """Per-decode-step aggregates of an ``LLMEngine``."""

    def __init__(self, log_interval: int = 0, stats_file: str = "", stats_interval: int = 100):
        super().__init__(log_interval, stats_file, stats_interval)
        self.steps = 0
        self._window = [0, 0, 0, 0.0, 0.0, 0.0]  # steps, rows, emitted, device_ms, host_ms, proposer_us

    @classmethod
    def from_env(cls) -> "Telemetry":
        return cls(_env_int("SUFFIX_HYBRID_LOG_INTERVAL", 0), os.environ.get("SUFFIX_HYBRID_STATS_FILE", "").strip(),
                   _env_int("SUFFIX_HYBRID_STATS_INTERVAL", 100))

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
        to_log, to_file = self.due(self.steps)
        if not (to_log or to_file):
            return
        rec = {"ts": time.time(), "step": self.steps, "method": engine.cfg.spec.method, "k": engine.k,
               "window_steps": w[0], "mean_accept_len": w[2] / w[1] if w[1] else 0.0,
               "device_ms_per_step": w[3] / w[0], "host_ms_per_step": w[4] / w[0],
               "proposer_us_per_step": w[5] / w[0], "running": len(engine.running), "waiting": len(engine.waiting),
               "prefilling": int(getattr(engine, "prefilling", None) is not None),
               "proposer": engine.proposer_stats()}
        self.write(rec, to_log, to_file)
        self._window = [0, 0, 0, 0.0, 0.0, 0.0]


class CallTelemetry(_Sink):
    """Per-call telemetry of a proposer object.

    ``after_call(ns)`` is called once per ``propose`` with the call's wall
    time.  The time goes to ``charge`` (the native proposer's running total);
    on due calls ``snapshot()`` is written as a record with a timestamp, and
    the writing time is charged as well.
    """

    def __init__(self, snapshot: Callable[[], dict], charge: Optional[Callable[[int], object]] = None,
                 log_interval: int = 100, stats_file: str = "", stats_interval: int = 100):
        super().__init__(log_interval, stats_file, stats_interval)
        self.snapshot = snapshot
        self.charge = charge or (lambda ns: None)
        self.calls = 0

    @classmethod
    def from_env(cls, snapshot, charge=None) -> "CallTelemetry":
        return cls(snapshot, charge, _env_int("SUFFIX_HYBRID_LOG_INTERVAL", 100),
                   os.environ.get("SUFFIX_HYBRID_STATS_FILE", "").strip(), _env_int("SUFFIX_HYBRID_STATS_INTERVAL", 100))

    def after_call(self, elapsed_ns: int) -> None:
        self.calls += 1
        self.charge(elapsed_ns)
        to_log, to_file = self.due(self.calls)
        if not (to_log or to_file):
            return
        t0 = time.perf_counter_ns()
        rec = dict(self.snapshot())
        rec["ts"] = time.time()
        self.write(rec, to_log, to_file)
        self.charge(time.perf_counter_ns() - t0)
