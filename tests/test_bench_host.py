"""Host-side pieces of bench.py that need no GPU."""
import importlib.util
import os

from conftest import ROOT


def load_bench():
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    m = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(m)
    return m


def test_clock_summary_parses_nvidia_smi_lines():
    b = load_bench()
    lines = ["0, 1965, 1965, 650.1, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
             "0, 1800, 1965, 990.0, 0x0000000000000004, Not Active, Not Active, Not Active, Active",
             "0, 1900, 1965, 900.0, 0x0000000000000000, Not Active, Not Active, Not Active, Not Active",
             "garbage"]
    s = b.summarize_clocks(lines)
    assert s["sm_mhz"] == 1900 and s["sm_max_mhz"] == 1965
    assert s["reasons"] == ["sw_power_cap"] and s["samples"] == 3


def test_peaks_read_measured_file():
    b = load_bench()
    peak, kind = b.peaks()
    assert peak > 1000 and kind in ("measured", "fallback")
