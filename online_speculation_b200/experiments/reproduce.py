"""One command for the reproduction pipeline: data, training, evaluation, infrastructure.

    python -m online_speculation_b200.experiments.reproduce --family arllm|dllm|both \\
        --stage prepare|train|eval|all --profile smoke|full --output-root runs/repro \\
        [--components quality passk distribution infra training] [--backend tabular|engine] \\
        [--limit N] [--dry-run] [--restart]

The driver turns the selection into a fixed list of commands of this package's own
entry points and runs it as a manifested suite (``suite_runner``): the plan's
fingerprint and the number of finished commands sit in
``<output-root>/<tag>/suite_manifest.json``, so re-running the same selection resumes
after the last finished command and a different selection for the same directory is
refused unless ``--restart``.

Stages and components:

* ``prepare`` writes the prompt set (``data/prompts.jsonl``): synthetic uniform-random
  token prompts whose answer is a fixed token suffix (no dataset download is
  possible offline; a real tokenised set in the same JSONL form can replace it with
  ``--prompts``);
* ``train`` runs GRPO (``training.grpo_run``, resumable ``checkpoint-N`` shards) for
  ``arllm``; the ``dllm`` family trains nothing here;
* ``eval`` runs, per component, ``quality`` (every method once per prompt, accuracy
  with Wilson intervals and the paired bootstrap against ``base``), ``passk`` (several
  draws, pass@k), ``distribution`` (samplers against exactly enumerable targets) and
  ``infra`` (the benchmark workloads: suffix-MH with speculation and conditional IS
  for ``arllm``, block diffusion for ``dllm``);
* ``all`` is prepare, train and eval.

``smoke`` keeps every command small enough for the CPU tabular oracle (``infra`` and
``train`` need a GPU and are left out of a smoke run unless named explicitly);
``full`` uses the engine backend on the Qwen2.5-1.5B shape.  The command layout
follows experiments/run_reproduction.py and experiments/arllm/run_arllm_suite.py.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

from .artifacts import write_json_atomic
from .suite_runner import run_manifested_commands

ROOT = Path(__file__).resolve().parents[2]
COMPONENTS = ("quality", "passk", "distribution", "infra", "training")
FAMILY_COMPONENTS = {"arllm": COMPONENTS, "dllm": ("infra",)}
GPU_COMPONENTS = ("infra", "training")
SMOKE_COMPONENTS = ("quality", "passk", "distribution")
PROFILES = {
    # prompts, prompt length, draws for pass@k, MH chains / runs of the audit, GRPO steps, bench steps
    "smoke": {"prompts": 4, "prompt_length": 8, "passk_draws": 4, "audit_chains": 600, "audit_runs": 60,
              "grpo_steps": 4, "grpo_model": "tiny", "bench_steps": 2, "is_prompts": 8, "vocab": 32},
    "full": {"prompts": 64, "prompt_length": 256, "passk_draws": 16, "audit_chains": 3000, "audit_runs": 300,
             "grpo_steps": 100, "grpo_model": "qwen2.5-1.5b", "bench_steps": 4, "is_prompts": 64, "vocab": 151936},
}


def write_prompts(path: Path, count: int, length: int, vocab: int, seed: int, answer=(0, 0)) -> None:
    """Synthetic prompt set in the runner's JSONL form; correct = the completion ends with ``answer``."""
    rng = np.random.default_rng(seed)
    path.parent.mkdir(parents=True, exist_ok=True)
    with path.open("w", encoding="utf-8") as handle:
        for i in range(count):
            ids = rng.integers(1, vocab - 1, size=length).tolist()
            handle.write(json.dumps({"id": f"prompt-{i}", "prompt_ids": ids, "answer": list(answer)}) + "\n")


def _stages(stage: str) -> tuple[str, ...]:
    return ("prepare", "train", "eval") if stage == "all" else (stage,)


def build_commands(args) -> list[list[str]]:
    prof = dict(PROFILES[args.profile])
    if args.limit is not None:
        prof["prompts"] = min(prof["prompts"], args.limit)
    out = Path(args.output_root) / args.tag
    py = sys.executable
    prompts = Path(args.prompts) if args.prompts else out / "data" / "prompts.jsonl"
    backend = args.backend or ("tabular" if args.profile == "smoke" else "engine")
    vocab = 32 if backend == "tabular" else prof["vocab"]
    commands: list[list[str]] = []
    stages = _stages(args.stage)
    families = ("arllm", "dllm") if args.family == "both" else (args.family,)
    if "prepare" in stages and not args.prompts:
        commands.append([py, "-m", "online_speculation_b200.experiments.reproduce", "prepare-data",
                         "--path", str(prompts), "--count", str(prof["prompts"]),
                         "--length", str(prof["prompt_length"]), "--vocab", str(vocab), "--seed", str(args.seed)])
    for family in families:
        chosen = [c for c in args.components if c in FAMILY_COMPONENTS[family]]
        fam = out / family
        if "train" in stages and family == "arllm" and "training" in chosen:
            commands.append([py, "-m", "online_speculation_b200.training.grpo_run", "--output", str(fam / "grpo"),
                             "--model", prof["grpo_model"], "--max-steps", str(prof["grpo_steps"]),
                             "--save-steps", str(max(1, prof["grpo_steps"] // 4)), "--resume", "auto",
                             "--seed", str(args.seed)])
        if "eval" not in stages:
            continue
        runner = [py, "-m", "online_speculation_b200.experiments.run", "--prompts", str(prompts), "--backend", backend,
                  "--vocab", str(vocab), "--seed", str(args.seed)]
        if family == "arllm" and "quality" in chosen:
            commands.append(runner + ["--methods", ",".join(args.methods), "--draws", "1", "--out",
                                      str(fam / "quality")])
        if family == "arllm" and "passk" in chosen:
            commands.append(runner + ["--methods", "base,conditional_is", "--draws", str(prof["passk_draws"]),
                                      "--out", str(fam / "passk")])
        if family == "arllm" and "distribution" in chosen:
            commands.append([py, "-m", "online_speculation_b200.experiments.distribution_audit", "--out",
                             str(fam / "distribution.json"), "--chains", str(prof["audit_chains"]),
                             "--runs", str(prof["audit_runs"]), "--seed", str(args.seed)])
        if "infra" in chosen:
            bench = [py, str(ROOT / "bench.py"), "--steps", str(prof["bench_steps"]), "--warmup", "3"]
            if family == "arllm":
                commands.append(bench + ["--json-out", str(fam / "infra_mh_spec.json")])
                commands.append(bench + ["--workload", "is", "--is-prompts", str(prof["is_prompts"]),
                                         "--json-out", str(fam / "infra_conditional_is.json")])
            else:
                commands.append(bench + ["--workload", "dllm", "--json-out", str(fam / "infra_block_diffusion.json")])
    return commands


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if argv[:1] == ["prepare-data"]:
        p = argparse.ArgumentParser(prog="reproduce prepare-data")
        p.add_argument("--path", required=True)
        p.add_argument("--count", type=int, required=True)
        p.add_argument("--length", type=int, required=True)
        p.add_argument("--vocab", type=int, required=True)
        p.add_argument("--seed", type=int, default=0)
        a = p.parse_args(argv[1:])
        write_prompts(Path(a.path), a.count, a.length, a.vocab, a.seed)
        print(json.dumps({"prompts": a.path, "count": a.count}))
        return 0
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.reproduce")
    p.add_argument("--family", choices=("arllm", "dllm", "both"), default="arllm")
    p.add_argument("--stage", choices=("prepare", "train", "eval", "all"), default="all")
    p.add_argument("--profile", choices=tuple(PROFILES), default="smoke")
    p.add_argument("--components", nargs="+", choices=COMPONENTS)
    p.add_argument("--methods", nargs="+", default=["base", "mh", "conditional_is"])
    p.add_argument("--backend", choices=("tabular", "engine"))
    p.add_argument("--prompts", help="an existing prompt JSONL (skips data preparation)")
    p.add_argument("--output-root", default="runs/reproduction")
    p.add_argument("--tag", default="reproduction")
    p.add_argument("--limit", type=int, help="at most this many prompts")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--restart", action="store_true")
    a = p.parse_args(argv)
    if a.components is None:
        a.components = list(SMOKE_COMPONENTS if a.profile == "smoke" else COMPONENTS)
    commands = build_commands(a)
    out = Path(a.output_root) / a.tag
    metadata = {"family": a.family, "stage": a.stage, "profile": a.profile, "components": sorted(a.components),
                "methods": a.methods, "seed": a.seed}
    manifest = run_manifested_commands(commands=commands, root=ROOT, manifest_path=out / "suite_manifest.json",
                                       metadata=metadata, dry_run=a.dry_run, restart=a.restart)
    if not a.dry_run:
        write_json_atomic(out / "reproduction_summary.json", {
            "status": manifest["status"], "commands": manifest["commands"],
            "results": sorted(str(p.relative_to(out)) for p in out.rglob("*.json")
                              if p.name not in ("suite_manifest.json", "reproduction_summary.json"))}, indent=2)
    print(json.dumps({"status": manifest["status"], "commands": len(commands),
                      "manifest": str(out / "suite_manifest.json")}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
