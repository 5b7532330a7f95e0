"""Reproduction driver (CPU): plan construction, smoke run on the tabular oracle, resume and refusal."""

import json

import pytest

from online_speculation_b200.experiments import reproduce


def test_plans_cover_the_selected_stages_and_components(tmp_path):
    argv = ["--family", "both", "--stage", "all", "--profile", "full", "--output-root", str(tmp_path), "--dry-run"]
    assert reproduce.main(argv) == 0
    manifest = json.loads((tmp_path / "reproduction" / "suite_manifest.json").read_text())
    text = "\n".join(manifest["commands"])
    for needle in ("prepare-data", "training.grpo_run", "experiments.run", "distribution_audit",
                   "--workload is", "--workload dllm"):
        assert needle in text
    assert manifest["status"] == "dry_run"


def test_smoke_pipeline_runs_resumes_and_refuses_other_plans(tmp_path):
    argv = ["--stage", "all", "--profile", "smoke", "--output-root", str(tmp_path), "--limit", "2"]
    assert reproduce.main(argv) == 0
    out = tmp_path / "reproduction"
    summary = json.loads((out / "arllm" / "quality" / "summary.json").read_text())
    assert set(summary["methods"]) == {"base", "mh", "conditional_is"}
    passk = json.loads((out / "arllm" / "passk" / "summary.json").read_text())
    assert "pass_at_k" in passk["methods"]["base"]
    assert json.loads((out / "arllm" / "distribution.json").read_text())["passed"]
    manifest = json.loads((out / "suite_manifest.json").read_text())
    assert manifest["status"] == "complete" and manifest["completed_commands"] == len(manifest["commands"])
    assert reproduce.main(argv) == 0                     # same plan: every command is skipped
    with pytest.raises(ValueError):
        reproduce.main(argv[:-2] + ["--limit", "3"])     # a different plan for the same directory
