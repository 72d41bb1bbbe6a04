"""CPU: bench.py's clock record keeps the samples drawn under load.

The sampler reads nvidia-smi's CSV (index, clocks.sm, clocks.max.sm,
power.draw, the active flag and four throttle reasons); idle samples taken
before and after the timed region (board power below half of the run's
highest sample) are left out of the median and of the reasons."""
import os
import sys
import tempfile

sys.path.insert(0, os.path.join(os.path.dirname(__file__), ".."))

import bench  # noqa: E402


class _Done:
    def terminate(self):
        pass

    def wait(self):
        pass


def _record(lines):
    s = bench.ClockSampler(0)
    fd, s.path = tempfile.mkstemp(suffix=".csv")
    with os.fdopen(fd, "w") as f:
        f.write("\n".join(lines) + "\n")
    s.proc = _Done()
    return s.stop()


def test_median_over_loaded_samples():
    idle = "0, 1965 MHz, 1965 MHz, 150.00 W, Not Active, Not Active, Not Active, Not Active, Not Active"
    busy = "0, {} MHz, 1965 MHz, 950.00 W, Active, Not Active, Not Active, Not Active, Active"
    clk = _record([idle, idle, busy.format(1700), busy.format(1750), busy.format(1800), idle])
    assert clk["sm_mhz"] == 1750
    assert clk["sm_max_mhz"] == 1965
    assert clk["samples"] == 3 and clk["samples_all"] == 6
    assert clk["reasons"] == ["sw_power_cap"]


def test_no_power_column_keeps_every_sample():
    line = "0, {} MHz, 1965 MHz, [N/A], Not Active, Not Active, Not Active, Not Active, Not Active"
    clk = _record([line.format(1900), line.format(1950), line.format(1965)])
    assert clk["sm_mhz"] == 1950 and clk["samples"] == 3 and clk["reasons"] == []
