"""bench.py's clock record during the timed region, read through NVML: the
sampler collects samples, reports the median SM clock and the maximum, and
names the clock-event reasons that were active.  Runs against a fake NVML
module (read-only queries only; no GPU, no settings touched)."""
import importlib.util
import os
import sys
import time
import types

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _fake_nvml(reasons_bits):
    m = types.ModuleType("pynvml")
    m.NVML_CLOCK_SM = 1
    m.nvmlClocksEventReasonHwSlowdown = 0x8
    m.nvmlClocksEventReasonHwThermalSlowdown = 0x40
    m.nvmlClocksEventReasonSwThermalSlowdown = 0x20
    m.nvmlClocksEventReasonSwPowerCap = 0x4
    clocks = iter([1965, 1900, 1965, 1965, 1800] + [1965] * 10000)
    m.nvmlInit = lambda: None

    def by_uuid(_):
        raise RuntimeError("no device with that uuid")

    m.nvmlDeviceGetHandleByUUID = by_uuid
    m.nvmlDeviceGetHandleByIndex = lambda i: ("gpu", i)
    m.nvmlDeviceGetClockInfo = lambda h, kind: next(clocks)
    m.nvmlDeviceGetMaxClockInfo = lambda h, kind: 1965
    m.nvmlDeviceGetCurrentClocksEventReasons = lambda h: reasons_bits
    return m


def _bench_module():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("bits,want", [(0x0, []), (0x4, ["sw_power_cap"]), (0x4 | 0x40, ["hw_thermal_slowdown", "sw_power_cap"])])
def test_clock_sampler_reads_nvml(monkeypatch, bits, want):
    monkeypatch.setitem(sys.modules, "pynvml", _fake_nvml(bits))
    bench = _bench_module()
    with bench.ClockSampler(0) as clk:
        time.sleep(0.08)
    s = clk.summary()
    assert s["source"] == "nvml"
    assert s["samples"] >= 3
    assert s["sm_max_mhz"] == 1965.0
    assert 1800.0 <= s["sm_mhz"] <= 1965.0
    assert s["reasons"] == want


def test_clock_sampler_without_nvml_reports_unsampled(monkeypatch):
    broken = types.ModuleType("pynvml")

    def fail():
        raise RuntimeError("NVML unavailable")

    broken.nvmlInit = fail
    monkeypatch.setitem(sys.modules, "pynvml", broken)
    monkeypatch.setenv("PATH", "")  # no nvidia-smi either
    bench = _bench_module()
    with bench.ClockSampler(0) as clk:
        time.sleep(0.05)
    s = clk.summary()
    assert s["samples"] == 0 and s["reasons"] == ["unsampled"]
