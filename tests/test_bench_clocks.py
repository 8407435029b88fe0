"""bench.py's clock sampler (CPU): nvidia-smi rows are kept only inside the
timed region's window, a region shorter than the sampling period still gets
the first samples after it began, and throttle reasons are collected."""
import datetime
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))


def _sampler_with_rows(rows):
    import bench
    s = bench.ClockSampler(0)
    fd, s.path = tempfile.mkstemp(suffix=".csv")
    with os.fdopen(fd, "w") as f:
        f.write("\n".join(rows) + "\n")
    s.proc = subprocess.Popen([sys.executable, "-c", "import time; time.sleep(30)"])
    return s


def _row(t, mhz, cap="Not Active"):
    stamp = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return f"{stamp}, 0, {mhz}, 1965, 900.0, 0x0, Not Active, Not Active, Not Active, {cap}"


def test_window_keeps_only_timed_samples():
    base = 1_700_000_000.0
    rows = [_row(base + 0.05 * i, 1900 if i < 10 else 1600, "Active" if i >= 10 else "Not Active")
            for i in range(20)]
    info = _sampler_with_rows(rows).stop((base + 0.5, base + 0.96))
    assert info["samples"] == 10 and info["sm_mhz"] == 1600.0
    assert info["sm_max_mhz"] == 1965.0 and info["reasons"] == ["sw_power_cap"]


def test_short_region_takes_first_samples_after_start():
    base = 1_700_000_000.0
    rows = [_row(base + 0.05 * i, 1800 + i) for i in range(6)]
    info = _sampler_with_rows(rows).stop((base + 0.101, base + 0.102))
    assert info["samples"] == 2 and info["sm_mhz"] == (1803 + 1804) / 2
    assert info["reasons"] == []
