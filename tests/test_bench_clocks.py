"""bench.py's clock sampler: samples inside the timed region (host wall-clock window, widened by
one sampling period) are the ones reported; reasons come from the NVML clock-event bits."""

import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def _sampler(rows):
    s = bench.ClockSampler(reader=None)
    s.samples = list(rows)  # (t, sm_mhz, max_mhz, power_w, util, reasons_mask)
    return s


def test_samples_inside_the_timed_window_are_reported():
    t0 = 1_800_000_000.0
    rows = [(t0 + 0.02 * i, 1965 if i < 10 or i >= 14 else 1700, 1965, 700.0, 100, 0x4 if 10 <= i < 14 else 0)
            for i in range(20)]
    c = _sampler(rows).stop((t0 + 0.2, t0 + 0.26))  # samples 10..13 within +-20 ms
    assert c["sampled"] == "timed region"
    assert c["sm_mhz"] == 1700 and c["reasons"] == ["sw_power_cap"] and c["sm_max_mhz"] == 1965


def test_no_sample_in_the_window_falls_back_to_loaded_samples():
    t0 = 1_800_000_000.0
    rows = [(t0 + 0.02 * i, 1965, 1965, 500.0, 100 if i % 2 else 0, 0) for i in range(6)]
    c = _sampler(rows).stop((t0 + 10.0, t0 + 10.01))
    assert c["sampled"].startswith("samples under load") and c["samples"] == 3 and c["reasons"] == []


def test_slowdown_bits_are_named():
    t0 = 1_800_000_000.0
    rows = [(t0, 1500, 1965, 900.0, 100, 0x8 | 0x40), (t0 + 0.02, 1500, 1965, 900.0, 100, 0x20)]
    c = _sampler(rows).stop((t0, t0 + 0.02))
    assert c["reasons"] == ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown"]


def test_reader_thread_collects_samples():
    import time

    s = bench.ClockSampler(reader=lambda: (1965, 1965, 600.0, 99, 0))
    time.sleep(0.1)
    c = s.stop()
    assert c["samples"] >= 2 and c["sm_mhz"] == 1965


def test_unsampled_without_a_reader():
    assert bench.ClockSampler(reader=None).stop((0.0, 1.0))["reasons"] == ["unsampled"]
