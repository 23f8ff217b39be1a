"""CPU: bench.py's clock sampler reports the lag-shifted window of its NVML samples (median
clock, every active clock-event reason by name, board power)."""
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, REPO)

import bench  # noqa: E402


def _sampler(samples, smax=1965.0):
    cs = bench.ClockSampler(0)
    cs.ok = True
    cs.smax = smax
    cs.samples = samples

    class _T:
        def join(self, timeout=None):
            return None

    cs.t = _T()
    return cs


def test_window_is_shifted_by_the_telemetry_lag(monkeypatch):
    monkeypatch.setattr(bench.time, "sleep", lambda s: None)
    t0 = 100.0
    lag = bench.ClockSampler.LAG_S
    # idle readings before the region's effect reaches NVML, loaded readings after the lag
    samples = [(t0 + 0.01 * i, 1965.0, 0x0, 250.0) for i in range(15)]
    samples += [(t0 + lag + 0.01 * i, 1100.0, 0x4, 900.0) for i in range(20)]
    cs = _sampler(samples)
    monkeypatch.setattr(bench.time, "monotonic", lambda: t0 + 0.2)  # the region ends at t0 + 0.2
    out = cs.stop(t0)
    assert out["sm_mhz"] == 1100.0
    assert out["reasons"] == ["sw_power_cap"]
    assert out["power_w"] == 900.0
    assert out["samples"] == 20


def test_all_reason_bits_are_named(monkeypatch):
    monkeypatch.setattr(bench.time, "sleep", lambda s: None)
    t0 = 10.0
    bits = 0x1 | 0x8 | 0x40 | 0x80
    samples = [(t0 + bench.ClockSampler.LAG_S + 0.01 * i, 900.0, bits, 700.0) for i in range(5)]
    cs = _sampler(samples)
    monkeypatch.setattr(bench.time, "monotonic", lambda: t0 + 0.05)
    out = cs.stop(t0)
    assert out["reasons"] == sorted(["gpu_idle", "hw_slowdown", "hw_thermal_slowdown", "hw_power_brake_slowdown"])


def test_short_region_falls_back_to_everything_it_may_cover(monkeypatch):
    monkeypatch.setattr(bench.time, "sleep", lambda s: None)
    t0 = 5.0
    samples = [(t0 + 0.01, 1500.0, 0x4, 600.0), (t0 + 0.02, 1400.0, 0x4, 650.0)]
    cs = _sampler(samples)
    monkeypatch.setattr(bench.time, "monotonic", lambda: t0 + 0.005)
    out = cs.stop(t0)
    assert out["samples"] == 2 and out["sm_mhz"] == 1450.0
