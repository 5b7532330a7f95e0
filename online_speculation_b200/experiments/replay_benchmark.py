"""Replay benchmarks: what reusing stored rollouts buys base replay and dynamic IS, at fixed budgets.

Two sections over the same prompts, seeds, lengths and candidate counts:

* ``replay`` -- base-candidate replay (truncated-IS history plus a fresh tail):
  ``fresh_only`` (no history: every candidate weight comes from fresh rollouts) against
  ``warm_replay`` (before each decision a history policy writes rollouts for the decision's
  candidate blocks into the replay store -- the cache build, timed apart -- and every
  candidate reuses up to ``max_history`` of them next to its fresh rollouts);
* ``dynamic_is`` -- defensive-mixture candidates with a variance-cost rollout budget:
  ``base_candidate_fixed`` (base candidates only, constant design statistics),
  ``replay_aware_fixed`` (an auxiliary proposal mixed into the candidates and a store
  prepared with history rollouts of the decision's candidates, constant statistics) and
  ``replay_aware_optimal`` (the same with the empirical variance-cost design statistics).

Every arm reports device and wall seconds, generated tokens per second, the rollouts it
drew fresh against those it reused from the store, the candidates' mean effective sample
size, and the mean reward of its outputs.  Any backend works: the exact tabular model on
the CPU (tests) or the engine backend on a GPU (``random:<preset>`` weights and
uniform-random prompts from the command line).

    python -m online_speculation_b200.experiments.replay_benchmark --output replay.json \\
        [--model random:qwen2.5-0.5b] [--section replay|dynamic_is|all] [--prompts 2] \\
        [--max-new-tokens 32] [--block-size 8] [--candidates 4]

Purpose and arm names of experiments/arllm/gsm8k_replay_benchmark.py and
experiments/arllm/gsm8k_dynamic_is_benchmark.py; the GSM8K data, verifier rewards and the
small-model history policy of those scripts are replaced by synthetic prompts, a
sequence-log-probability reward and a hotter policy of the same backend.
"""

from __future__ import annotations

import argparse
import json
from collections.abc import Callable, Sequence
from pathlib import Path
from typing import Any

import numpy as np

from ..arllm.config import BaseReplayConfig, SamplingConfig
from ..arllm.replay import BehaviorPolicy, BehaviorRegistry, InMemoryReplayStore
from ..shared.rng import SeedStream
from .rollout_infra import counter_delta, measure


def _estimates(steps) -> list:
    return [c.estimate for st in steps for c in st.candidates]


def _summary(name: str, results, t: dict, reward: Callable, prompts, before, after) -> dict:
    est = _estimates([st for r in results for st in r.steps])
    tokens = sum(len(r.token_ids) for r in results)
    ess = [float(e.history_ess) + float(e.fresh_ess) for e in est]
    return {"name": name, "online": {
        "telemetry": t, "main_model": counter_delta(before, after), "output_tokens": tokens,
        "output_tokens_per_second": tokens / t["device_seconds"] if t["device_seconds"] else 0.0,
        "decisions": sum(len(r.steps) for r in results),
        "history_rollouts_reused": int(sum(e.history_count for e in est)),
        "fresh_rollouts": int(sum(e.fresh_count for e in est)),
        "reserve_records_written": int(sum(r.reserve_records_written for r in results)),
        "mean_candidate_ess": float(np.mean(ess)) if ess else 0.0,
        "mean_output_reward": float(np.mean([reward(p, r.token_ids) for p, r in zip(prompts, results)])),
    }}


def replay_arms(backend, *, prompts: Sequence[tuple], length: int, block: int, candidates: int, seed: int,
                reward: Callable, history: int = 4, fresh: int = 2, history_temperature: float = 1.3) -> list[dict]:
    """Base replay with and without a warm store.

    Every decision first draws its candidate blocks (the step's own seed stream); the warm
    arm then writes ``history`` rollouts per candidate from the history policy into the
    store (the cache build, timed and counted apart from the online work), and the step
    runs on those frozen candidates, reusing up to ``history`` stored rollouts each.
    """
    from ..arllm.algorithms.base_replay import base_replay_step
    from ..arllm.algorithms.conditional_is import sample_candidates
    from ..arllm.replay import ReplayKey, ReplaySampleRequest, sample_replay_records

    out = []
    sampling = SamplingConfig()
    for name in ("fresh_only", "warm_replay"):
        warm = name == "warm_replay"
        cfg = BaseReplayConfig(candidate_count=candidates, block_size=block, total_length=length,
                               reward_temperature=0.5, max_history_per_candidate=history if warm else 0,
                               fresh_rollouts=fresh)
        hist_policy = BehaviorPolicy.for_backend(backend, SamplingConfig(temperature=history_temperature),
                                                 label="history")
        snap = getattr(backend, "snapshot", lambda: None)
        build = {"wall_seconds": 0.0, "device_seconds": 0.0, "records": 0}

        def one(i, prompt):
            seeds = SeedStream(SeedStream(seed).derive("replay", i))
            registry, store = BehaviorRegistry([hist_policy]), InMemoryReplayStore()
            generated: tuple = ()
            steps = []
            while len(generated) < length:
                k = len(steps)
                b = min(block, length - len(generated))
                rollout = length - len(generated) - b
                cands = sample_candidates(backend, tuple(prompt) + generated, candidates, b, sampling, seeds, k)
                if warm and rollout > 0:
                    reqs = [ReplaySampleRequest(ReplayKey(tuple(prompt), generated, c.token_ids, "reward"), rollout,
                                                seeds.derive("history", k, j, h), f"history:{i}:{k}:{j}:{h}")
                            for j, c in enumerate(cands) for h in range(history)]
                    recs, t = measure(lambda: sample_replay_records(hist_policy, reqs, reward))
                    for r in recs:
                        store.add_evaluation(r)
                    build["wall_seconds"] += t["wall_seconds"]
                    build["device_seconds"] += t["device_seconds"]
                    build["records"] += len(recs)
                st = base_replay_step(base_backend=backend, registry=registry, store=store, prompt=prompt,
                                      generated_prefix=generated, config=cfg, base_sampling=sampling, reward=reward,
                                      reward_version="reward", seeds=seeds, step_index=k, candidate_samples=cands)
                steps.append(st)
                generated += tuple(st.selected.token_ids)
            return _Result(generated, tuple(steps), 0)

        before = snap()
        results, t = measure(lambda: [one(i, p) for i, p in enumerate(prompts)])
        t = {k: t[k] - build[k] for k in t}                 # online time excludes the cache build
        rec = _summary(name, results, t, reward, prompts, before, snap())
        rec["cache_build"] = build
        out.append(rec)
    return out


class _Result:
    def __init__(self, token_ids, steps, reserve_records_written):
        self.token_ids, self.steps, self.reserve_records_written = token_ids, steps, reserve_records_written


def dynamic_is_arms(backend, *, prompts: Sequence[tuple], length: int, block: int, candidates: int, seed: int,
                    reward: Callable, history: int = 4, budget: float = 16.0) -> list[dict]:
    """Dynamic IS arms (:func:`~online_speculation_b200.experimental.arllm.dynamic_is.run_dynamic_is_arm`);
    the replay-aware arms' history preparation is the cache build, timed apart."""
    from ..experimental.arllm.dynamic_is import DYNAMIC_ARMS, run_dynamic_is_arm

    out = []
    for name in DYNAMIC_ARMS:
        snap = getattr(backend, "snapshot", lambda: None)
        build = {"wall_seconds": 0.0, "device_seconds": 0.0, "records": 0}

        def timed(make):
            recs, t = measure(make)
            build["wall_seconds"] += t["wall_seconds"]
            build["device_seconds"] += t["device_seconds"]
            build["records"] += len(recs)
            return recs

        def run():
            return [run_dynamic_is_arm(backend, p, arm=name, candidate_count=candidates, block_size=block,
                                       total_length=length, reward=reward,
                                       seeds=SeedStream(SeedStream(seed).derive("dynamic", i)), history=history,
                                       rollout_budget=budget, prepare=timed)
                    for i, p in enumerate(prompts)]

        before = snap()
        results, t = measure(run)
        t = {k: t[k] - build[k] for k in t}
        rec = _summary(name, results, t, reward, prompts, before, snap())
        rec["cache_build"] = build
        draws = [c.draw for r in results for st in r.steps for c in st.candidates]
        rec["online"]["auxiliary_candidates"] = sum(d.source == "auxiliary" for d in draws)
        out.append(rec)
    return out


def run_benchmark(backend, *, prompts: Sequence[tuple], section: str = "all", length: int = 32, block: int = 8,
                  candidates: int = 4, seed: int = 20260812, reward: Callable | None = None) -> dict:
    reward = reward or (lambda _p, y: 0.0)
    report: dict[str, Any] = {"workload": {"prompts": len(prompts), "prompt_tokens": [len(p) for p in prompts],
                                           "max_new_tokens": length, "block_size": block,
                                           "candidate_count": candidates, "seed": seed}}
    if section in ("replay", "all"):
        report["replay"] = replay_arms(backend, prompts=prompts, length=length, block=block, candidates=candidates,
                                       seed=seed, reward=reward)
    if section in ("dynamic_is", "all"):
        report["dynamic_is"] = dynamic_is_arms(backend, prompts=prompts, length=length, block=block,
                                               candidates=candidates, seed=seed, reward=reward)
    return report


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.replay_benchmark")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--model", default="random:qwen2.5-0.5b", help="random:<preset> or a local checkpoint directory")
    p.add_argument("--section", choices=("replay", "dynamic_is", "all"), default="all")
    p.add_argument("--prompts", type=int, default=2)
    p.add_argument("--prompt-tokens", type=int, default=64)
    p.add_argument("--max-new-tokens", type=int, default=32)
    p.add_argument("--block-size", type=int, default=8)
    p.add_argument("--candidates", type=int, default=4)
    p.add_argument("--kv-cache-gb", type=float, default=8.0)
    p.add_argument("--seed", type=int, default=20260812)
    a = p.parse_args(argv)

    from ..arllm.backends.loader import LoadedModel
    from ..arllm.rewards import SequenceLogProbabilityReward

    backend = LoadedModel(a.model, {"runtime": {"kv_cache_gb": a.kv_cache_gb, "max_batch_size": 64,
                                                "max_sequence_tokens": a.prompt_tokens + 2 * a.max_new_tokens + 64}},
                          "base").backend
    try:
        rng = np.random.default_rng(a.seed)
        prompts = [tuple(int(t) for t in rng.integers(0, backend.vocab_size, a.prompt_tokens))
                   for _ in range(a.prompts)]
        report = run_benchmark(backend, prompts=prompts, section=a.section, length=a.max_new_tokens,
                               block=a.block_size, candidates=a.candidates, seed=a.seed,
                               reward=SequenceLogProbabilityReward(backend, coefficient=0.5))
    finally:
        backend.close()
    report.update(model=a.model, data="synthetic uniform-random prompts"
                  + (", random-init weights" if a.model.startswith("random:") else ""))
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(report, indent=2))
    print(json.dumps({"output": str(a.output), "seconds": {
        arm["name"]: round(arm["online"]["telemetry"]["device_seconds"], 3)
        for sec in ("replay", "dynamic_is") for arm in report.get(sec, [])}}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
