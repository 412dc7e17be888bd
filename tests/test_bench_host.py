"""Host-side pieces of bench.py that need no GPU: the CPU binding of a rank (HostBinding) and the choice of the
roofline's peak. Without NVML (or without a GPU) the binding leaves the process where it was, and lending the CPUs
back for the CPU baselines restores exactly the original set."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def test_host_binding_keeps_or_narrows_the_cpu_set_and_lends_it_back():
    before = os.sched_getaffinity(0)
    h = bench.HostBinding(0)
    try:
        bound = os.sched_getaffinity(0)
        assert bound <= before  # never widens
        s = h.summary()
        assert s["cpus_total"] == len(before)
        assert s["cpus_near_gpu"] is None or s["cpus_near_gpu"] == len(bound)
        with h.everywhere():
            assert os.sched_getaffinity(0) == before
        assert os.sched_getaffinity(0) == bound
    finally:
        os.sched_setaffinity(0, before)


def test_roofline_peaks_pick_the_sustained_figure_under_the_power_cap():
    peaks, peak, kind, burst, sust, capped = bench.roofline_peaks({"reasons": ["sw_power_cap"]}, False)
    assert capped and kind == "sustained" and peak == sust
    peaks, peak, kind, burst, sust, capped = bench.roofline_peaks({"reasons": []}, False)
    assert not capped and kind == "burst" and peak == burst
    peaks, peak, kind, burst, sust, capped = bench.roofline_peaks({"reasons": []}, True)
    assert kind == "sustained"
