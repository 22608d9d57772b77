"""Host-side parts of bench.py, on CPU: the clock sampler that records the
SM clock and the clock-event reasons during the timed region, against a fake
NVML binding (read-only queries; nothing here touches a GPU setting)."""
from __future__ import annotations

import importlib.util
import sys
import time
import types
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("oxf_bench", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _fake_nvml(clocks, reasons, fail_init=False):
    """A stand-in pynvml: SM clocks and reason bitmasks served in turn."""
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    state = {"i": 0}

    def init():
        if fail_init:
            raise RuntimeError("NVML unavailable")

    def clock(h, kind):
        assert kind == 1
        v = clocks[min(state["i"], len(clocks) - 1)]
        return v

    def event_reasons(h):
        v = reasons[min(state["i"], len(reasons) - 1)]
        state["i"] += 1
        return v

    m.nvmlInit = init
    m.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    m.nvmlDeviceGetClockInfo = clock
    m.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    m.nvmlDeviceGetCurrentClocksEventReasons = event_reasons
    return m


def test_clock_sampler_reads_nvml(bench, monkeypatch):
    clocks = [1400, 1350, 1380, 1330, 1360]
    reasons = [0x4, 0x4, 0x0, 0x4 | 0x20, 0x4]  # sw_power_cap, one sw_thermal_slowdown
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(clocks, reasons))
    # as on a GPU host: every device visible (torch maps CUDA device 0 to NVML index 0)
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES", raising=False)
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.3)
    out = s.stop()
    assert out["source"] == "nvml"
    assert out["samples"] >= 5
    assert out["sm_max_mhz"] == 1965.0
    assert 1330 <= out["sm_mhz"] <= 1400
    assert out["reasons"] == ["sw_power_cap", "sw_thermal_slowdown"]


def test_clock_sampler_falls_back_without_nvml(bench, monkeypatch):
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml([1], [0], fail_init=True))
    calls = []

    def smi(self):
        calls.append(1)
        return ["0", "1500", "1965", "700.5", "0x4", "Not Active", "Not Active", "Not Active",
                "Active"]

    monkeypatch.setattr(bench.ClockSampler, "_smi", smi)
    s = bench.ClockSampler(0)
    s.start()
    time.sleep(0.3)
    out = s.stop()
    assert out["source"] == "nvidia-smi" and calls
    assert out["sm_mhz"] == 1500.0 and out["reasons"] == ["sw_power_cap"]
