"""bench.py's clock sampler against a fake nvidia-smi (no GPU): start() returns once sampling
runs, only samples taken inside the timed region count, and the median SM clock, the maximum
clock and the active throttle reasons are read from the CSV."""
from __future__ import annotations

import os
import stat
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

FAKE = """#!/usr/bin/env python3
import sys, time
time.sleep(0.3)                                  # start-up delay, as the real tool has
print("0, 1000, 1965, 500.0, Not Active, Not Active, Not Active, Not Active", flush=True)  # before the region
i = 0
while True:
    time.sleep(0.05)
    cap = "Active" if i == 2 else "Not Active"
    print(f"0, {1100 + 10 * (i % 3)}, 1965, 990.5, Not Active, Not Active, Not Active, {cap}", flush=True)
    i += 1
"""


def test_clock_sampler_with_fake_nvidia_smi(tmp_path, monkeypatch):
    fake = tmp_path / "nvidia-smi"
    fake.write_text(FAKE)
    fake.chmod(fake.stat().st_mode | stat.S_IXUSR | stat.S_IXGRP | stat.S_IXOTH)
    monkeypatch.setenv("PATH", f"{tmp_path}{os.pathsep}{os.environ['PATH']}")
    sys.path.insert(0, ROOT)
    import bench
    c = bench.Clocks(0)
    t0 = time.time()
    c.start()
    assert time.time() - t0 >= 0.25          # waited for the first sample
    time.sleep(0.5)                          # the "timed region"
    r = c.stop()
    assert r["samples"] >= 3                 # the pre-region sample is not among them
    assert r["sm_max_mhz"] == 1965.0
    assert 1100.0 <= r["sm_mhz"] <= 1120.0
    assert r["reasons"] == ["sw_power_cap"]


def test_clock_sampler_without_nvidia_smi(tmp_path, monkeypatch):
    monkeypatch.setenv("PATH", str(tmp_path))  # no nvidia-smi anywhere
    sys.path.insert(0, ROOT)
    import bench
    c = bench.Clocks(0)
    c.start()
    r = c.stop()
    assert r["sm_mhz"] is None and r["samples"] == 0
