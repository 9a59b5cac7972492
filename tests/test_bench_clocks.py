"""bench.py's clock sampler: samples are read from nvidia-smi's CSV and those inside the timed
region (host wall-clock window, widened by one sampling period) are the ones reported."""

import datetime
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


class _FakeProc:
    def __init__(self, out):
        self.out = out

    def terminate(self):
        pass

    def communicate(self, timeout=None):
        return self.out, ""


def _line(t, mhz, util, power_cap):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    cap = "Active" if power_cap else "Not Active"
    return f"{ts}, {mhz}, 1965, 700.0, {util}, Not Active, Not Active, Not Active, {cap}"


def _sampler(lines):
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.proc = _FakeProc("\n".join(lines) + "\n")
    return s


def test_samples_inside_the_timed_window_are_reported():
    t0 = 1_800_000_000.0
    lines = [_line(t0 + 0.05 * i, 1965 if i < 10 or i >= 14 else 1700, 100, 10 <= i < 14) for i in range(20)]
    c = _sampler(lines).stop((t0 + 0.55, t0 + 0.65))  # samples 10..13 within +-50 ms
    assert c["sampled"] == "timed region"
    assert c["sm_mhz"] == 1700 and c["reasons"] == ["sw_power_cap"] and c["sm_max_mhz"] == 1965


def test_no_sample_in_the_window_falls_back_to_loaded_samples():
    t0 = 1_800_000_000.0
    lines = [_line(t0 + 0.05 * i, 1965, 100 if i % 2 else 0, False) for i in range(6)]
    c = _sampler(lines).stop((t0 + 10.0, t0 + 10.01))
    assert c["sampled"].startswith("samples under load") and c["samples"] == 3 and c["reasons"] == []


def test_unsampled_without_nvidia_smi():
    s = bench.ClockSampler.__new__(bench.ClockSampler)
    s.proc = None
    assert s.stop((0.0, 1.0))["reasons"] == ["unsampled"]
