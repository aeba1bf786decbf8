"""bench.py's clock sampler against a fake NVML (read-only queries, no GPU).

The sampler must yield at least one sample for a timed region of a few
milliseconds and report the throttle reasons the driver rejects runs for.
"""
from __future__ import annotations

import sys
import time
import types

import bench


def fake_nvml(reason_mask: int, sm_mhz: int = 1965) -> types.ModuleType:
    nv = types.ModuleType("pynvml")
    nv.NVML_CLOCK_SM = 1
    nv.nvmlInit = lambda: None
    nv.nvmlDeviceGetHandleByUUID = lambda uuid: "h"
    nv.nvmlDeviceGetHandleByIndex = lambda i: "h"
    nv.nvmlDeviceGetCurrentClocksEventReasons = lambda h: reason_mask
    nv.nvmlDeviceGetClockInfo = lambda h, kind: sm_mhz
    nv.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    nv.nvmlDeviceGetPowerUsage = lambda h: 812_000
    return nv


def test_short_region_still_sampled(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", fake_nvml(0x1 | 0x4, sm_mhz=1800))
    with bench.ClockSampler(0) as clocks:
        time.sleep(0.002)
    s = clocks.summary()
    assert s["source"] == "nvml" and s["samples"] >= 1
    assert s["sm_mhz"] == 1800 and s["sm_max_mhz"] == 1965 and s["power_w_max"] == 812.0
    assert s["reasons"] == ["sw_power_cap"]  # GPU-idle bit is not a slowdown


def test_slowdown_reasons_reported(monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", fake_nvml(0x8 | 0x20 | 0x40))
    with bench.ClockSampler(0) as clocks:
        time.sleep(0.05)
    s = clocks.summary()
    assert s["samples"] >= 2
    assert s["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_no_nvml_no_smi_gives_none(monkeypatch):
    nv = fake_nvml(0)

    def fail():
        raise RuntimeError("no driver")

    nv.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    monkeypatch.setattr(bench.subprocess, "Popen", lambda *a, **k: (_ for _ in ()).throw(OSError("absent")))
    with bench.ClockSampler(0) as clocks:
        pass
    assert clocks.summary() is None
