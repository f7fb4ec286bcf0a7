"""Sample SM clocks, power and clock-event (throttle) reasons during a timed region.

A background thread polls NVML (nvidia-ml-py) every `period_ms`; without
NVML it falls back to `nvidia-smi -lms`.  Only reads are issued: no clock,
power or mode setting is changed.
"""
from __future__ import annotations

import os
import statistics
import subprocess
import tempfile
import threading

_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
           "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
           "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
_REASON_NAMES = {"sw_power_cap": "SwPowerCap", "hw_slowdown": "HwSlowdown", "sw_thermal_slowdown": "SwThermalSlowdown",
                 "hw_thermal_slowdown": "HwThermalSlowdown", "hw_power_brake_slowdown": "HwPowerBrakeSlowdown"}


def _visible_indices(gpus):
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [int(v) for v in vis.split(",") if v.strip().isdigit()]
        return [ids[g] for g in gpus if g < len(ids)] if gpus is not None else ids
    return list(gpus) if gpus is not None else [0]


class ClockSampler:
    def __init__(self, period_ms: int = 20, gpus=None):
        self.period_ms = period_ms
        self.gpus = gpus
        self.samples = []  # (sm_mhz, max_mhz, power_w, reasons set)
        self._stop = threading.Event()
        self._thread = None
        self.proc = None
        self.out = None
        self.mode = None

    def start(self) -> None:
        try:
            import pynvml

            pynvml.nvmlInit()
            bits_of = {n: getattr(pynvml, "nvmlClocksEventReason" + v) for n, v in _REASON_NAMES.items()}
            handles = [pynvml.nvmlDeviceGetHandleByIndex(i) for i in _visible_indices(self.gpus or [0])]
            self.mode = "nvml"

            def loop():
                while not self._stop.is_set():
                    for h in handles:
                        try:
                            sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
                            pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                            bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        except Exception:
                            continue
                        self.samples.append((float(sm), float(mx), pw,
                                             {n for n, b in bits_of.items() if bits & b}))
                    self._stop.wait(self.period_ms / 1000.0)

            self._thread = threading.Thread(target=loop, daemon=True)
            self._thread.start()
            return
        except Exception:
            self.mode = None
        try:
            self.out = tempfile.TemporaryFile(mode="w+")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={_FIELDS}", "--format=csv,noheader,nounits",
                                          f"-lms={max(self.period_ms, 100)}"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
            self.mode = "nvidia-smi"
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read_smi(self, gpus):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.out.seek(0)
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.read().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
                if gpus is not None and idx not in gpus:
                    continue
                sm, mx, pw = float(parts[1]), float(parts[2]), float(parts[3])
            except ValueError:
                continue
            self.samples.append((sm, mx, pw, {n for n, v in zip(names, parts[5:9]) if v.lower() == "active"}))

    def stop(self, gpus=None) -> dict:
        if self.mode == "nvml":
            self._stop.set()
            self._thread.join(timeout=5)
        elif self.mode == "nvidia-smi" and self.proc is not None:
            self._read_smi(gpus)
        else:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no clock source (NVML / nvidia-smi)"]}
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = set()
        for s in self.samples:
            reasons |= s[3]
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples),
                "power_w_max": max(s[2] for s in self.samples), "samples": len(self.samples),
                "source": self.mode, "reasons": sorted(reasons)}
