"""Run sampling methods over a prompt set with resumable results and a summary.

    python -m online_speculation_b200.experiments.run \\
        --methods base,mh,conditional_is --draws 4 --out results/run1 \\
        [--prompts prompts.jsonl] [--backend tabular|engine] [--model qwen2.5-1.5b] \\
        [--reward verifier|sequence_logprob|zeros] [--set max_new_tokens=64 ...]

Prompts come from a JSONL file (``{"id": ..., "prompt_ids": [...], "answer": ...}``)
or are synthetic.  Every (method, prompt, draw) record is appended to
``records.jsonl`` as soon as it finishes and skipped when the run is resumed;
``summary.json`` holds per-method accuracy with Wilson intervals, pass@k
(from the draws), mean reward and the paired clustered bootstrap of every
method against ``base``.  A manifest pins the run's configuration: resuming
with different settings is refused.

Reference behaviour: experiments/arllm/gsm8k_reproduction.py (per-method
runner), experiments/shared/{artifacts,statistics}.py (records and reports).
"""

from __future__ import annotations

import argparse
import json
import time
from dataclasses import asdict
from pathlib import Path

from .artifacts import append_jsonl, apply_config_overrides, indexed_records, json_fingerprint, load_jsonl, \
    write_json_atomic
from .methods import RUNNABLE_AR_METHODS, MethodSettings, run_ar_method
from .statistics import clustered_paired_binary_difference, estimated_pass_at_k, wilson_interval


def _load_prompts(path: str | None, count: int, length: int, vocab: int, seed: int) -> list[dict]:
    if path:
        rows = load_jsonl(Path(path))
        for r in rows:
            if "id" not in r or "prompt_ids" not in r:
                raise ValueError("prompt records need 'id' and 'prompt_ids'")
        return rows
    import numpy as np

    rng = np.random.default_rng(seed)
    return [{"id": f"synthetic-{i}", "prompt_ids": rng.integers(1, vocab - 1, size=length).tolist(), "answer": None}
            for i in range(count)]


def _build_backend(kind: str, model: str, vocab: int, max_len: int, seed: int):
    if kind == "tabular":
        from ..arllm.backends.tabular import TabularBackend

        return TabularBackend.per_position_logits(vocab, max_len, seed=seed, prompt_length=0)
    import torch

    from ..api import build_runner
    from ..engine.backend import EngineBackend

    torch.cuda.set_device(0)
    return EngineBackend(build_runner(model, seed=seed), max_batch=64)


def _build_reward(kind: str, backend):
    if kind == "zeros":
        return lambda prompt, y: sum(t == 0 for t in y) / max(1, len(y))
    if kind == "sequence_logprob":
        from ..arllm.rewards import SequenceLogProbabilityReward

        return SequenceLogProbabilityReward(backend, coefficient=0.5)
    raise ValueError(f"unknown reward {kind!r}")


def _correct(record_tokens, answer) -> bool:
    if answer is None:
        return False
    if isinstance(answer, list):
        return list(record_tokens[-len(answer):]) == answer if answer else False
    return str(answer) in " ".join(map(str, record_tokens))


def summarize(records: list[dict], methods: list[str], draws: int, seed: int = 0) -> dict:
    out: dict = {"methods": {}}
    for m in methods:
        rs = [r for r in records if r["method"] == m]
        if not rs:
            continue
        n = len(rs)
        c = sum(bool(r["correct"]) for r in rs)
        entry = {"records": n, "accuracy": c / n, "wilson_95": wilson_interval(c, n),
                 "mean_seconds": sum(r["seconds"] for r in rs) / n}
        rewards = [r["reward"] for r in rs if r.get("reward") is not None]
        if rewards:
            entry["mean_reward"] = sum(rewards) / len(rewards)
        by_prompt: dict = {}
        for r in rs:
            by_prompt.setdefault(r["prompt"], []).append(bool(r["correct"]))
        if draws > 1 and all(len(v) == draws for v in by_prompt.values()):
            entry["pass_at_k"] = {k: sum(estimated_pass_at_k(sum(v), draws, k) for v in by_prompt.values())
                                  / len(by_prompt) for k in range(1, draws + 1)}
        out["methods"][m] = entry
    if "base" in out["methods"]:
        base = [dict(r, cluster=r["prompt_index"]) for r in records if r["method"] == "base"]
        for m in out["methods"]:
            if m == "base":
                continue
            other = [dict(r, cluster=r["prompt_index"]) for r in records if r["method"] == m]
            try:
                out["methods"][m]["vs_base"] = clustered_paired_binary_difference(
                    other, base, cluster_key="cluster", outcome_key="correct", seed=seed, replicates=2000)
            except ValueError:
                pass
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.run")
    p.add_argument("--methods", default="base,mh,conditional_is")
    p.add_argument("--draws", type=int, default=1)
    p.add_argument("--out", required=True)
    p.add_argument("--prompts")
    p.add_argument("--synthetic-prompts", type=int, default=4)
    p.add_argument("--prompt-length", type=int, default=8)
    p.add_argument("--backend", choices=("tabular", "engine"), default="tabular")
    p.add_argument("--model", default="qwen2.5-1.5b")
    p.add_argument("--vocab", type=int, default=32)
    p.add_argument("--reward", choices=("zeros", "sequence_logprob"), default="zeros")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--set", action="append", default=[], help="method setting override key=value")
    p.add_argument("--restart", action="store_true")
    a = p.parse_args(argv)
    methods = [m.strip() for m in a.methods.split(",") if m.strip()]
    for m in methods:
        if m not in RUNNABLE_AR_METHODS:
            raise SystemExit(f"method {m!r} is not runnable here; choose from {', '.join(RUNNABLE_AR_METHODS)}")
    settings_dict = apply_config_overrides({"settings": asdict(MethodSettings())},
                                           [f"settings.{s}" for s in a.set])["settings"]
    settings = MethodSettings(**settings_dict)
    out = Path(a.out)
    manifest = {"methods": methods, "draws": a.draws, "prompts": a.prompts, "synthetic": a.synthetic_prompts,
                "prompt_length": a.prompt_length, "backend": a.backend, "model": a.model, "vocab": a.vocab,
                "reward": a.reward, "seed": a.seed, "settings": settings_dict}
    mpath = out / "manifest.json"
    if mpath.is_file() and not a.restart:
        old = json.loads(mpath.read_text(encoding="utf-8"))
        if old.get("fingerprint") != json_fingerprint(manifest):
            raise SystemExit(f"{mpath} was written with different settings; pass --restart to overwrite")
    elif a.restart and (out / "records.jsonl").is_file():
        (out / "records.jsonl").unlink()
    write_json_atomic(mpath, {**manifest, "fingerprint": json_fingerprint(manifest)}, indent=2)
    prompts = _load_prompts(a.prompts, a.synthetic_prompts, a.prompt_length, a.vocab, a.seed)
    backend = _build_backend(a.backend, a.model, a.vocab, a.prompt_length + settings.max_new_tokens + 1, a.seed)
    reward = _build_reward(a.reward, backend)
    rpath = out / "records.jsonl"
    done = indexed_records(load_jsonl(rpath), key=lambda r: (r["method"], r["prompt"], r["draw"]))
    for m in methods:
        for i, pr in enumerate(prompts):
            for d in range(a.draws):
                if (m, pr["id"], d) in done:
                    continue
                t0 = time.perf_counter()
                res = run_ar_method(m, backend, pr["prompt_ids"], settings, seed=a.seed * 1_000_003 + 7919 * i + d,
                                    reward=reward)
                rec = {"method": m, "prompt": pr["id"], "prompt_index": i, "draw": d,
                       "token_ids": list(res.token_ids), "reward": float(reward(tuple(pr["prompt_ids"]),
                                                                                res.token_ids)),
                       "correct": _correct(res.token_ids, pr.get("answer")), "seconds": time.perf_counter() - t0,
                       "diagnostics": json.loads(json.dumps(res.diagnostics, default=float))}
                append_jsonl(rpath, rec)
                done[(m, pr["id"], d)] = rec
    records = load_jsonl(rpath)
    write_json_atomic(out / "summary.json", summarize(records, methods, a.draws, a.seed), indent=2)
    print(json.dumps({"records": len(records), "summary": str(out / "summary.json")}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
