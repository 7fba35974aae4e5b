"""bench.py's clock sampler against a stand-in NVML module (no GPU): samples
are taken only while the timed region is marked active, the clock-event
reason bits decode to their names, and a region shorter than the sampling
interval still gets one sample, taken just after it and labelled as such."""
from __future__ import annotations

import sys
import time
import types

import pytest

import bench


class FakeNvml(types.ModuleType):
    NVML_CLOCK_SM = 1

    def __init__(self, clock=1965, reasons=0):
        super().__init__("pynvml")
        self.clock = clock
        self.reasons = reasons
        self.calls = 0

    def nvmlInit(self):
        pass

    def nvmlDeviceGetHandleByUUID(self, uuid):
        return "gpu"

    def nvmlDeviceGetHandleByIndex(self, i):
        return "gpu"

    def nvmlDeviceGetClockInfo(self, h, kind):
        self.calls += 1
        return self.clock

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        return 1965

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.reasons


@pytest.fixture
def fake(monkeypatch):
    nv = FakeNvml()
    monkeypatch.setitem(sys.modules, "pynvml", nv)
    return nv


def test_samples_only_while_active(fake):
    c = bench.ClockSampler(0)
    c.start()
    time.sleep(0.05)  # idle before the region: no samples
    assert c.rows == []
    fake.clock = 1800
    c.active = True
    time.sleep(0.05)
    c.active = False
    n = len(c.rows)
    fake.clock = 300  # idle after the region: not sampled
    time.sleep(0.03)
    out = c.stop()
    assert n > 0 and out["samples"] == n
    assert out["sm_mhz"] == 1800.0 and out["sm_max_mhz"] == 1965.0
    assert out["reasons"] == [] and "timed region only" in out["source"]


def test_reason_bits_decode(fake):
    fake.reasons = 0x4 | 0x40 | 0x1  # sw_power_cap, hw_thermal_slowdown, gpu idle (not reported)
    c = bench.ClockSampler(0)
    c.start()
    c.active = True
    time.sleep(0.03)
    out = c.stop()
    assert out["reasons"] == ["hw_thermal_slowdown", "sw_power_cap"]


def test_short_region_gets_one_sample(fake):
    c = bench.ClockSampler(0)
    c.start()
    c.active = True  # stopped before the sampling thread sees it
    c.active = False
    c.rows.clear()
    out = c.stop()
    assert out["samples"] == 1 and out["sm_mhz"] == 1965.0
    assert "shorter than 2 ms" in out["source"]
