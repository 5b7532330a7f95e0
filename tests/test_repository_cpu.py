"""Repository hygiene: the files the user documentation and the profile summaries cite exist,
every profile summary carries the command that made it, and the driver-facing entry points keep
their contracts."""

import ast
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "online_speculation_b200")
# reference-side paths cited for parity (they name the reference project's files, not ours)
REFERENCE_PREFIXES = ("src/", "experiments/arllm/", "experiments/dllm/", "experiments/shared/", "online-speculation/",
                      "configs/", "ablation/")


def _cited_files(markdown: str):
    text = open(os.path.join(ROOT, markdown), encoding="utf-8").read()
    for tok in re.findall(r"`([^`\s]+)`", text):
        path = tok.split("::")[0]
        if re.search(r"\.(py|cu|cuh|h|cpp|md)$", path) and not path.startswith(REFERENCE_PREFIXES):
            yield path


def _expand(path: str):
    """Brace alternatives (``a/{b,c}.py``) as separate paths."""
    m = re.search(r"\{([^{}]*)\}", path)
    if m is None:
        return [path]
    return [q for alt in m.group(1).split(",") for q in _expand(path[:m.start()] + alt + path[m.end():])]


@pytest.mark.parametrize("markdown", ["README.md"] + sorted(os.path.relpath(p, ROOT) for p in
                                                          glob.glob(os.path.join(ROOT, "profiles", "*.md"))))
def test_cited_files_exist(markdown):
    here = os.path.dirname(os.path.join(ROOT, markdown))
    missing = [q for p in _cited_files(markdown) for q in _expand(p)
               if not any(glob.glob(os.path.join(base, q)) for base in (ROOT, PKG, here))]
    assert not missing, f"{markdown} cites files that do not exist: {missing}"


def test_profile_summaries_carry_their_commands():
    files = sorted(glob.glob(os.path.join(ROOT, "profiles", "*.md")))
    assert files
    for f in files:
        text = open(f, encoding="utf-8").read()
        assert re.search(r"^\s+(python|ncu|timeout|CUDA_VISIBLE_DEVICES)\b", text, re.M), f"{f} names no command"


def test_entry_points_keep_their_contracts():
    entry = ast.parse(open(os.path.join(ROOT, "__graft_entry__.py"), encoding="utf-8").read())
    names = {n.name for n in entry.body if isinstance(n, ast.FunctionDef)}
    assert {"build", "smoke"} <= names
    bench = open(os.path.join(ROOT, "bench.py"), encoding="utf-8").read()
    for flag in ("--gpus", "--steps", "--warmup", "--impl", "--workload"):
        assert flag in bench, flag
    for key in ('"metric"', '"value"', '"ms_per_step"', '"e2e"', '"gpu_launches"', '"clocks"', '"vs_baseline"'):
        assert key in bench, key


def test_every_module_imports_without_a_gpu():
    import importlib
    import pkgutil

    import online_speculation_b200 as pkg

    failed = []
    for mod in pkgutil.walk_packages(pkg.__path__, prefix="online_speculation_b200."):
        if mod.name.endswith("__main__"):
            continue
        try:
            importlib.import_module(mod.name)
        except Exception as err:                # noqa: BLE001 - collected for the report
            failed.append(f"{mod.name}: {type(err).__name__}: {err}")
    assert not failed, failed


@pytest.mark.parametrize("workload", ["grpo", "dllm"])
def test_unavailable_reference_arms_report_without_a_gpu(workload):
    import json
    import subprocess
    import sys

    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          workload], capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unavailable"]
