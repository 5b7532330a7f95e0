"""Experiment layer: statistics, artifacts, resumable suites, method registry and runner (CPU)."""

import json
import math
import sys

import pytest

from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.experiments import artifacts as A
from online_speculation_b200.experiments import statistics as S
from online_speculation_b200.experiments.methods import (AR_DEFAULT_METHODS, AR_METHODS, DLLM_METHODS,
                                                         RUNNABLE_AR_METHODS, MethodSettings, method_spec,
                                                         run_ar_method)
from online_speculation_b200.experiments.run import main as run_main
from online_speculation_b200.experiments.suite_runner import run_manifested_commands


def test_statistics():
    lo, hi = S.wilson_interval(8, 10)
    assert lo == pytest.approx(0.4901625, abs=1e-6) and hi == pytest.approx(0.9433178, abs=1e-6)
    assert S.estimated_pass_at_k(2, 5, 1) == pytest.approx(0.4)
    assert S.estimated_pass_at_k(2, 5, 4) == 1.0
    assert S.estimated_pass_at_k(0, 5, 3) == 0.0
    assert S.quantile([3, 1, 2, 4], 0.5) == 2.5
    a = S.bootstrap_mean_interval([1, 2, 3, 4, 5], seed=3, replicates=500)
    assert a == S.bootstrap_mean_interval([1, 2, 3, 4, 5], seed=3, replicates=500) and a[0] < 3 < a[1]
    left = [{"c": i, "ok": i % 2 == 0} for i in range(10) for _ in range(2)]
    right = [{"c": i, "ok": False} for i in range(10) for _ in range(2)]
    r = S.clustered_paired_binary_difference(left, right, cluster_key="c", outcome_key="ok", seed=0, replicates=300)
    assert r["difference"] == pytest.approx(0.5) and r["clustered_bootstrap_95"][0] > 0
    with pytest.raises(ValueError):
        S.clustered_paired_binary_difference(left, right[:-1], cluster_key="c", outcome_key="ok", seed=0)
    p, q = {"a": 0.5, "b": 0.5}, {"a": 1.0}
    assert S.total_variation_distance(p, q) == pytest.approx(0.5)
    assert S.jensen_shannon_bits(p, p) == 0.0 and 0 < S.jensen_shannon_bits(p, q) <= 1.0
    d = S.bootstrap_answer_distance({0: ["x", "y"]}, {0: ["x", "x"]}, [0], replicates=50)
    assert 0 <= d["mean_total_variation_bootstrap_95"][0] <= d["mean_total_variation_bootstrap_95"][1] <= 1


def test_artifacts(tmp_path):
    A.write_json_atomic(tmp_path / "a.json", {"x": 1})
    assert json.loads((tmp_path / "a.json").read_text()) == {"x": 1}
    assert A.json_fingerprint({"b": 1, "a": 2}) == A.json_fingerprint({"a": 2, "b": 1})
    p = tmp_path / "r.jsonl"
    A.append_jsonl(p, {"k": 1})
    A.append_jsonl(p, {"k": 2})
    with p.open("a") as f:
        f.write('{"k": 3')           # an interrupted append
    assert [r["k"] for r in A.load_jsonl(p)] == [1, 2]
    with pytest.raises(ValueError):
        A.indexed_records([{"k": 1, "v": 1}, {"k": 1, "v": 2}], key=lambda r: r["k"])
    cfg = {"a": {"b": 1, "c": "x"}}
    assert A.apply_config_overrides(cfg, ["a.b=3", "a.c=[1, 2]"]) == {"a": {"b": 3, "c": [1, 2]}}
    with pytest.raises(KeyError):
        A.apply_config_overrides(cfg, ["a.missing=1"])
    assert A.parse_override_value("none") is None and A.parse_override_value("hello") == "hello"
    h1 = A.cached_file_sha256(tmp_path / "a.json", cache_directory=tmp_path / "cache")
    assert h1 == A.file_sha256(tmp_path / "a.json") == A.cached_file_sha256(tmp_path / "a.json",
                                                                         cache_directory=tmp_path / "cache")


def test_suite_runner_resumes_and_refuses_changed_plans(tmp_path):
    marker = tmp_path / "count.txt"
    cmd = [sys.executable, "-c", f"p=r'{marker}';import os;n=int(open(p).read()) if os.path.exists(p) else 0;"
                                 f"open(p,'w').write(str(n+1))"]
    fail = [sys.executable, "-c", "raise SystemExit(3)"]
    man = tmp_path / "m.json"
    with pytest.raises(Exception):
        run_manifested_commands(commands=[cmd, fail], root=tmp_path, manifest_path=man, metadata={"suite": "t"})
    m = json.loads(man.read_text())
    assert m["status"] == "failed" and m["completed_commands"] == 1
    with pytest.raises(Exception):
        run_manifested_commands(commands=[cmd, fail], root=tmp_path, manifest_path=man, metadata={"suite": "t"})
    assert marker.read_text() == "1"      # the completed command was not re-run
    with pytest.raises(ValueError):
        run_manifested_commands(commands=[cmd], root=tmp_path, manifest_path=man, metadata={"suite": "t"})
    m = run_manifested_commands(commands=[cmd], root=tmp_path, manifest_path=man, metadata={"suite": "t"},
                                restart=True)
    assert m["status"] == "complete" and marker.read_text() == "2"


def test_method_registry_and_runnables():
    assert "mh" in AR_METHODS and "base" in AR_DEFAULT_METHODS and "trajectory_power_mh" in DLLM_METHODS
    assert method_spec("arllm", "conditional_is_small_proposal").requires_proposal
    with pytest.raises(ValueError):
        method_spec("arllm", "nope")
    b = TabularBackend.per_position_logits(16, 12, seed=1, prompt_length=2)
    reward = lambda p, y: sum(t == 0 for t in y) / len(y)
    s = MethodSettings(max_new_tokens=6, block_size=2, candidates=2, rollouts=2, best_of=3, particles=2)
    for name in RUNNABLE_AR_METHODS:
        out = run_ar_method(name, b, (3, 4), s, seed=5, reward=reward)
        assert len(out.token_ids) == 6, name
    with pytest.raises(NotImplementedError):
        run_ar_method("rl_sample", b, (3, 4), s, seed=5, reward=reward)


def test_runner_cli_resumes(tmp_path):
    args = ["--methods", "base,reward_mh", "--draws", "2", "--out", str(tmp_path / "r"), "--set",
            "max_new_tokens=6", "--set", "block_size=2", "--synthetic-prompts", "3"]
    assert run_main(args) == 0
    recs = (tmp_path / "r" / "records.jsonl").read_text().splitlines()
    assert len(recs) == 2 * 3 * 2
    summary = json.loads((tmp_path / "r" / "summary.json").read_text())
    assert set(summary["methods"]) == {"base", "reward_mh"} and "vs_base" in summary["methods"]["reward_mh"]
    assert run_main(args) == 0
    assert len((tmp_path / "r" / "records.jsonl").read_text().splitlines()) == 12
    with pytest.raises(SystemExit):
        run_main(args[:-1] + ["4"])
    assert math.isfinite(summary["methods"]["base"]["mean_seconds"])
