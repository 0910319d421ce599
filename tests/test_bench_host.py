"""Host logic of bench.py that needs no GPU: the clock record it attaches to every line (nvidia-smi samples taken
during the timed region: median SM clock, the throttle reasons seen, a reading right after a region too short for
the sampler)."""
import os
import sys
import tempfile

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402


class _Done:
    def terminate(self):
        pass

    def wait(self):
        return 0


def _handle(text):
    f = tempfile.NamedTemporaryFile("w", suffix=".csv", delete=False)
    f.write(text)
    f.flush()
    return _Done(), f


def test_clocks_parse_samples():
    rows = ["0, 1965, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, Not Active",
            "0, 1800, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
            "0, 1965, 1965, 710.0, 0x0, Not Active, Not Active, Not Active, Not Active",
            "1, 900, 1965, 100.0, 0x0, Active, Not Active, Not Active, Not Active"]  # another GPU: ignored
    rec = bench.clocks_stop(_handle("\n".join(rows) + "\n"), [0])
    assert rec["sm_mhz"] == 1965.0 and rec["sm_max_mhz"] == 1965.0 and rec["samples"] == 3
    assert rec["reasons"] == ["sw_power_cap"] and rec["gpus"] == [0] and "note" not in rec


def test_clocks_reasons_across_ranks():
    rows = ["0, 1965, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, Not Active",
            "1, 1500, 1965, 900.0, 0x40, Not Active, Not Active, Active, Not Active"]
    rec = bench.clocks_stop(_handle("\n".join(rows) + "\n"), [0, 1])
    assert rec["samples"] == 2 and rec["reasons"] == ["sw_thermal_slowdown"] and rec["gpus"] == [0, 1]


def test_clocks_without_sampler():
    assert bench.clocks_stop((None, None), [0]) is None
