"""CPU test of the power monitor against a fake nvidia-smi stream (no GPU is read or changed)."""

import sys

import pytest

from online_speculation_b200.utils.power import PowerMonitor

FAKE = ("import sys, time\n"
        "for w in (100.0, 200.0, 300.0):\n"
        "    print(f'{w}, 50, 1000, 40', flush=True)\n"
        "    time.sleep(0.05)\n"
        "print('[N/A], [N/A], 1, 1', flush=True)\n"
        "time.sleep(5)\n")


def test_summary_of_a_streamed_run():
    mon = PowerMonitor(interval_seconds=0.05, command=[sys.executable, "-c", FAKE]).start()
    import time

    time.sleep(0.6)
    out = mon.stop()
    assert out["samples"] == 3
    assert out["mean_power_watts"] == pytest.approx(200.0) and out["peak_power_watts"] == 300.0
    assert out["mean_utilization_percent"] == 50.0 and out["peak_temperature_c"] == 40.0
    assert 0 < out["gpu_power_integral_wh"] < 300.0 * 0.6 / 3600
    assert out["monitor_error"] and "unparsed" in out["monitor_error"]


def test_missing_tool_does_not_raise():
    out = PowerMonitor(command=["/nonexistent/nvidia-smi"]).start().stop()
    assert out["samples"] == 0 and out["mean_power_watts"] is None and out["monitor_error"]
    with pytest.raises(ValueError):
        PowerMonitor(interval_seconds=0)


def test_trace_ranges_nest_and_switch_off():
    import torch

    from online_speculation_b200.utils.tracing import set_tracing, trace_range, tracing_enabled

    with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CPU]) as prof:
        with trace_range("outer.phase"):
            with trace_range("inner.phase"):
                torch.ones(4).sum()
    names = {e.name for e in prof.events()}
    assert {"outer.phase", "inner.phase"} <= names
    set_tracing(False)
    try:
        assert not tracing_enabled()
        with trace_range("ignored"):
            pass
    finally:
        set_tracing(True)
