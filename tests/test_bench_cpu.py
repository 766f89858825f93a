"""bench.py's host-side bookkeeping, without a GPU: the algorithmic byte counts
the headline is computed from, and the clock record parser (timed window,
median, throttle reasons)."""
from __future__ import annotations

import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_c2_algorithmic_bytes():
    bench.set_rows(8192)
    assert bench.FWD_BYTES == 536_903_680          # read a + read b + write d
    assert bench.BWD_BYTES == 805_404_672          # read a + read b + RMW grad_a + RMW grad_b
    assert bench.STEP_BYTES == 1_342_308_352
    bench.set_rows(4096)
    assert bench.FWD_BYTES == 4096 * 8192 * 8 + 4096 * 4
    bench.set_rows(8192)


class _Done:
    def terminate(self):
        pass

    def wait(self):
        return 0


def _clocks_with(rows, tmp_path):
    c = bench.Clocks(0)
    c.proc = _Done()
    with open(c.file.name, "w") as f:
        for r in rows:
            f.write(", ".join(r) + "\n")
    return c


def _row(t, mhz, power_cap="Not Active", thermal="Not Active"):
    ts = datetime.datetime.fromtimestamp(t).strftime("%Y/%m/%d %H:%M:%S.%f")[:-3]
    return [ts, "0", str(mhz), "1965", "700.0", "0x0", "Not Active", "Not Active", thermal, power_cap]


def test_clock_record_window_median_and_reasons(tmp_path):
    t0 = 1_800_000_000.0
    rows = [_row(t0 - 5, 345), _row(t0 + 0.1, 1900), _row(t0 + 0.3, 1700, power_cap="Active"),
            _row(t0 + 0.5, 1800), _row(t0 + 9, 300, thermal="Active")]
    clk = _clocks_with(rows, tmp_path).stop(t0, t0 + 0.6)
    assert clk["samples"] == 3                      # idle samples outside the window are dropped
    assert clk["sm_mhz"] == 1800.0 and clk["sm_max_mhz"] == 1965.0
    assert clk["reasons"] == ["sw_power_cap"]      # the thermal sample lies outside the window


def test_clock_record_without_samples(tmp_path):
    clk = _clocks_with([], tmp_path).stop(0.0, 1.0)
    assert clk["samples"] == 0 and clk["reasons"] == ["no samples"]
