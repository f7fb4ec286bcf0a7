"""Background GPU monitor (SUFFIX_HYBRID_GPU_MON=<seconds>): one JSON line per interval with each visible
GPU's SM clock, power, temperature, memory in use and active clock-event (throttle) reasons, to
SUFFIX_HYBRID_GPU_MON_FILE or the log.  Read-only NVML queries: no clock, power or mode is changed.
(The reference's monitor reads AMD hwmon, gpu_mon.py; this one reads NVML.)
"""
from __future__ import annotations

import json
import logging
import os
import threading
import time
from typing import Optional

logger = logging.getLogger(__name__)

_REASONS = {"sw_power_cap": "SwPowerCap", "hw_slowdown": "HwSlowdown", "sw_thermal_slowdown": "SwThermalSlowdown",
            "hw_thermal_slowdown": "HwThermalSlowdown", "hw_power_brake_slowdown": "HwPowerBrakeSlowdown"}


def sample(nvml, handles) -> list:
    rows = []
    bits = {n: getattr(nvml, "nvmlClocksEventReason" + v, 0) for n, v in _REASONS.items()}
    for i, h in handles:
        try:
            mem = nvml.nvmlDeviceGetMemoryInfo(h)
            active = nvml.nvmlDeviceGetCurrentClocksEventReasons(h)
            rows.append({"gpu": i, "sm_mhz": nvml.nvmlDeviceGetClockInfo(h, nvml.NVML_CLOCK_SM),
                         "power_w": round(nvml.nvmlDeviceGetPowerUsage(h) / 1000.0, 1),
                         "temp_c": nvml.nvmlDeviceGetTemperature(h, nvml.NVML_TEMPERATURE_GPU),
                         "mem_used_gib": round(mem.used / 2 ** 30, 2),
                         "reasons": sorted(n for n, b in bits.items() if b and active & b)})
        except Exception as exc:  # a query can fail on a busy device: report it and keep sampling
            rows.append({"gpu": i, "error": type(exc).__name__})
    return rows


class GpuMonitor:
    def __init__(self, interval_s: float, path: Optional[str] = None, nvml=None):
        self.interval_s, self.path = interval_s, path
        self._nvml = nvml
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    @classmethod
    def from_env(cls) -> Optional["GpuMonitor"]:
        raw = os.environ.get("SUFFIX_HYBRID_GPU_MON", "").strip()
        if not raw:
            return None
        return cls(float(raw), os.environ.get("SUFFIX_HYBRID_GPU_MON_FILE") or None)

    def _handles(self):
        nv = self._nvml
        n = nv.nvmlDeviceGetCount()
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        ids = [int(v) for v in vis.split(",") if v.strip().isdigit()] if vis else list(range(n))
        return [(i, nv.nvmlDeviceGetHandleByIndex(i)) for i in ids if i < n]

    def start(self) -> bool:
        if self._nvml is None:
            try:
                import pynvml

                pynvml.nvmlInit()
                self._nvml = pynvml
            except Exception as exc:
                logger.warning("GPU monitor disabled: %s", exc)
                return False
        handles = self._handles()

        def loop():
            while not self._stop.is_set():
                line = json.dumps({"t": round(time.time(), 3), "gpus": sample(self._nvml, handles)})
                if self.path:
                    with open(self.path, "a") as fh:
                        fh.write(line + "\n")
                else:
                    logger.info("gpu_mon %s", line)
                self._stop.wait(self.interval_s)

        self._thread = threading.Thread(target=loop, name="gpu_mon", daemon=True)
        self._thread.start()
        return True

    def stop(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=5)
