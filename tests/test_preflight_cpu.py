"""CPU tests of the environment preflight (report layout, stage selection, failing checks)."""

import json

import pytest

from online_speculation_b200.utils import preflight as pf


def test_report_layout_and_failure_propagation():
    runners = {"inference": lambda: [("ok", True, "x"), ("bad", False, "y")], "checkpoints": lambda: [("ok", True, "")]}
    rep = pf.preflight(["inference", "checkpoints"], runners)
    assert rep["stages"]["inference"]["passed"] is False and rep["stages"]["checkpoints"]["passed"] is True
    assert rep["passed"] is False
    assert rep["stages"]["inference"]["checks"][1] == {"check": "bad", "passed": False, "detail": "y"}
    json.dumps(rep)
    with pytest.raises(ValueError):
        pf.preflight(["nope"], runners)


def test_real_checks_run_on_this_machine():
    rep = pf.preflight(["inference", "checkpoints", "training"])
    names = [c["check"] for c in rep["stages"]["inference"]["checks"]]
    assert "torch >= 2.9" in names and "a CUDA device is visible" in names
    assert all(isinstance(c["passed"], bool) for s in rep["stages"].values() for c in s["checks"])


def test_version_comparison():
    assert pf._version_at_least("2.11.0+cu128", (2, 9))
    assert not pf._version_at_least("2.8.1", (2, 9))
    assert pf._version_at_least("10.0", (2, 9))
