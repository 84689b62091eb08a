"""The bench's NVML clock sampler, against a fake NVML (no GPU).

The sampler must keep only the samples taken inside the timed region, report
their median SM clock, and name every clock-event reason seen there (a
throttled run is rejected on exactly these names).  It only reads: the fake
has no setter, so any attempt to change a clock would fail here.
"""
from __future__ import annotations

import time

import bench


class FakeNvml:
    NVML_CLOCK_SM = 1
    nvmlClocksEventReasonGpuIdle = 0x1
    nvmlClocksEventReasonApplicationsClocksSetting = 0x2
    nvmlClocksEventReasonSwPowerCap = 0x4
    nvmlClocksEventReasonHwSlowdown = 0x8
    nvmlClocksEventReasonSwThermalSlowdown = 0x20
    nvmlClocksEventReasonHwThermalSlowdown = 0x40
    nvmlClocksEventReasonHwPowerBrakeSlowdown = 0x80

    def __init__(self, timeline):
        # timeline(t) -> (sm_mhz, power_mw, reason_mask) at host time t
        self.timeline = timeline
        self.inited = 0

    def nvmlInit(self):
        self.inited += 1

    def nvmlShutdown(self):
        self.inited -= 1

    def nvmlDeviceGetHandleByPciBusId(self, bus):
        assert bus == "00000000:1b:00.0"
        return "h"

    def nvmlDeviceGetHandleByIndex(self, i):
        return "h"

    def nvmlDeviceGetMaxClockInfo(self, h, kind):
        assert kind == self.NVML_CLOCK_SM
        return 1965

    def nvmlDeviceGetClockInfo(self, h, kind):
        return self.timeline(time.perf_counter())[0]

    def nvmlDeviceGetPowerUsage(self, h):
        return self.timeline(time.perf_counter())[1]

    def nvmlDeviceGetCurrentClocksEventReasons(self, h):
        return self.timeline(time.perf_counter())[2]


def _run(timeline, busy, total=0.25):
    nv = FakeNvml(timeline)
    s = bench.NvmlSampler(pci_bus_id="00000000:1b:00.0", interval=0.002, nvml=nv)
    s.start()
    time.sleep(total)
    out = s.stop(busy)
    assert nv.inited == 0  # shut down again
    return out


def test_only_samples_inside_the_window_count():
    t0 = time.perf_counter()
    w = (t0 + 0.08, t0 + 0.16)

    def timeline(t):
        if w[0] <= t <= w[1]:
            return 1400, 990_000, 0x4  # under load: power-capped
        return 1965, 120_000, 0x1  # idle

    out = _run(timeline, w)
    assert out["samples_in_window"] >= 5
    assert out["sm_mhz"] == 1400 and out["sm_max_mhz"] == 1965
    assert out["reasons"] == ["sw_power_cap"]  # idle is never reported
    assert out["power_w_max"] == 990.0


def test_hardware_slowdown_inside_the_window_is_named():
    t0 = time.perf_counter()
    w = (t0 + 0.05, t0 + 0.2)

    def timeline(t):
        if w[0] <= t <= w[1]:
            return 1100, 700_000, 0x8 | 0x40
        return 1965, 100_000, 0

    out = _run(timeline, w)
    assert out["reasons"] == ["hw_slowdown", "hw_thermal_slowdown"]
    assert out["sm_mhz"] == 1100


def test_window_shorter_than_the_interval_falls_back_to_the_nearest_sample():
    t0 = time.perf_counter()
    w = (t0 + 0.1, t0 + 0.1000001)
    out = _run(lambda t: (1800, 500_000, 0), w)
    assert out["samples"] == 1 and out["sm_mhz"] == 1800
