"""Dev-mode argv splice and the NVML GPU monitor (against a fake NVML)."""
import json
import time
import types

import pytest

from vllm_suffix_hybrid_b200.serve import dev_args
from vllm_suffix_hybrid_b200.utils import gpu_mon


def test_splice_forms():
    argv = ["--model", "toy", "--k", "5", "--no-graphs", "--port=9000", "--k", "7"]
    out = dev_args.splice(argv, [["--k", 3], "--async-scheduling", ["--no-graphs", None], ["--port", "8001"]])
    assert out == ["--model", "toy", "--k", "3", "--port", "8001", "--async-scheduling"]
    with pytest.raises(ValueError):
        dev_args.splice(argv, [["--model", "other"]])
    with pytest.raises(ValueError):
        dev_args.splice(argv, ["k"])


def test_apply_archives_the_file(tmp_path, monkeypatch):
    f = tmp_path / "dev_args.json"
    f.write_text(json.dumps([["--max-num-seqs", 8]]))
    argv = ["--model", "toy"]
    assert dev_args.apply(argv, str(f)) is None  # gate off
    monkeypatch.setenv("SUFFIX_HYBRID_DEV_ARGS", "1")
    assert dev_args.apply(argv, str(f)) == [["--max-num-seqs", 8]]
    assert argv == ["--model", "toy", "--max-num-seqs", "8"]
    assert not f.exists() and (tmp_path / "dev_args.last.json").exists()


def test_gpu_monitor_with_fake_nvml(tmp_path):
    class Mem:
        used = 3 * 2 ** 30

    fake = types.SimpleNamespace(
        NVML_CLOCK_SM=0, NVML_TEMPERATURE_GPU=0, nvmlClocksEventReasonSwPowerCap=4,
        nvmlClocksEventReasonHwSlowdown=8, nvmlClocksEventReasonSwThermalSlowdown=32,
        nvmlClocksEventReasonHwThermalSlowdown=64, nvmlClocksEventReasonHwPowerBrakeSlowdown=128,
        nvmlDeviceGetCount=lambda: 2, nvmlDeviceGetHandleByIndex=lambda i: i,
        nvmlDeviceGetMemoryInfo=lambda h: Mem(), nvmlDeviceGetCurrentClocksEventReasons=lambda h: 4,
        nvmlDeviceGetClockInfo=lambda h, c: 1800, nvmlDeviceGetPowerUsage=lambda h: 700000,
        nvmlDeviceGetTemperature=lambda h, t: 55)
    rows = gpu_mon.sample(fake, [(0, 0), (1, 1)])
    assert rows[0] == {"gpu": 0, "sm_mhz": 1800, "power_w": 700.0, "temp_c": 55, "mem_used_gib": 3.0,
                       "reasons": ["sw_power_cap"]}
    path = tmp_path / "mon.jsonl"
    mon = gpu_mon.GpuMonitor(0.01, str(path), nvml=fake)
    assert mon.start()
    time.sleep(0.1)
    mon.stop()
    lines = path.read_text().splitlines()
    assert lines and len(json.loads(lines[0])["gpus"]) == 2
