"""Rollout-infrastructure ablations on one fixed workload: what each accelerator buys, measured.

Two sections, each a list of arms that share the model, prompts, seeds, output length and
algorithm budgets, so only the accelerator differs:

* ``decode``: plain sampling against rollout-reuse speculation (the engine backend's token
  tree, tiered by batch size).  A history phase fills the tree (timed and counted on its
  own, so the offline cost stays visible), then evaluation batches of shrinking size run
  -- the long tail where drafting pays.  Besides tokens/s and the draft counters, every arm
  reports the fraction of evaluation requests whose tokens equal the plain arm's.  The
  verification keeps the sampled law; with the same uniforms it reproduces the plain draws
  as far as the two forward shapes give the same logits, which holds for the peaked laws of
  a trained model but not for the near-flat laws of random-init weights, where bf16
  differences move inverse-CDF draws by a few token ids.
* ``algorithm``: conditional IS with and without speculation, and the SMC rollout forest
  with and without reservoir reuse; each reports output tokens/s and its rollout counts.
* ``reuse``: reward MH against a verifier with a controlled delay (``--verifier-delay``
  seconds per exact reward): the standard chain, the prefetched chain (the next proposals
  are generated while the reward of the current one is computed; same decisions, so the
  same chain), and the delayed-acceptance chain (a cheap surrogate screens proposals and
  only survivors pay for the exact reward).  Each reports wall seconds, exact reward
  evaluations and whether its chain equals the standard one (the purpose of
  experiments/arllm/benchmark_is_mh_reuse.py).

Device work is bracketed by ``torch.cuda.synchronize`` and timed with CUDA events (wall
time is recorded beside them).  Model weights are random (``random:<preset>``) or a local
checkpoint through the backend loader; with random weights the reward is the completion's
scaled log-probability under the base model (no tokenizer or dataset is needed).

    python -m online_speculation_b200.experiments.rollout_infra --output infra.json \\
        [--model random:qwen2.5-0.5b] [--section decode|algorithm|all] [--prompts 2] \\
        [--max-new-tokens 64] [--batch-sizes 4,2,1] [--draft-tokens 8] [--verifier-delay 0.05]

Purpose and arm layout of experiments/arllm/benchmark_rollout_infra.py; the record keys
(``cache_build``, ``online``, ``draft_cache``) follow it so summaries read both.
"""

from __future__ import annotations

import argparse
import json
import platform
import time
from collections.abc import Callable, Sequence
from dataclasses import asdict, is_dataclass
from pathlib import Path
from typing import Any

import numpy as np

from ..arllm.acceleration import ActiveBatchSpeculationConfig, SpeculationTier
from ..arllm.config import ConditionalISConfig, SamplingConfig
from ..arllm.types import GenerationRequest, SequenceSample
from ..shared.rng import SeedStream


def _numbers(snapshot: Any) -> dict[str, float]:
    if snapshot is None:
        return {}
    if is_dataclass(snapshot) and not isinstance(snapshot, type):
        snapshot = asdict(snapshot)
    return {k: v for k, v in dict(snapshot).items() if isinstance(v, (int, float)) and not isinstance(v, bool)}


def counter_delta(before: Any, after: Any) -> dict[str, float]:
    """Numeric counters of ``after`` minus those of ``before`` (snapshots as dataclasses or dicts)."""
    a, b = _numbers(before), _numbers(after)
    return {k: b[k] - a.get(k, 0) for k in b}


def measure(call: Callable[[], Any]) -> tuple[Any, dict[str, float]]:
    """Run ``call`` between device synchronisations; wall and CUDA-event seconds."""
    try:
        import torch

        cuda = torch.cuda.is_available()
    except ImportError:                                    # pragma: no cover - torch is a dependency
        cuda = False
    if cuda:
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
    t0 = time.perf_counter()
    out = call()
    if cuda:
        end.record()
        torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    return out, {"wall_seconds": wall, "device_seconds": start.elapsed_time(end) / 1e3 if cuda else wall}


def history_batches(prompts: Sequence[tuple], *, count: int, length: int, sampling: SamplingConfig,
                    seeds: SeedStream) -> list[list[GenerationRequest]]:
    return [[GenerationRequest(p, length, sampling, seeds.derive("infra", "history", i, d),
                               f"infra:history:prompt:{i}:draw:{d}") for d in range(count)]
            for i, p in enumerate(prompts)]


def evaluation_batches(prompts: Sequence[tuple], *, batch_sizes: Sequence[int], length: int,
                       sampling: SamplingConfig, seeds: SeedStream) -> list[list[GenerationRequest]]:
    return [[GenerationRequest(p, length, sampling, seeds.derive("infra", "evaluation", i, stage, d),
                               f"infra:evaluation:prompt:{i}:stage:{stage}:draw:{d}") for d in range(size)]
            for i, p in enumerate(prompts) for stage, size in enumerate(batch_sizes)]


def _run(backend, batches) -> list[SequenceSample]:
    out: list[SequenceSample] = []
    for b in batches:
        out.extend(backend.sample_batch(b))
    return out


def _tree_snapshot(backend) -> Any:
    snap = getattr(backend, "draft_cache_snapshot", None)
    return snap() if callable(snap) else None


def decode_arm(backend, *, name: str, speculative: bool, history: Sequence[Sequence[GenerationRequest]],
               evaluation: Sequence[Sequence[GenerationRequest]]) -> tuple[dict, dict[str, tuple]]:
    """One decode arm on a fresh backend: history phase (speculative arms only), then evaluation."""
    before = getattr(backend, "snapshot", lambda: None)()
    if speculative:
        hist, hist_t = measure(lambda: _run(backend, history))
    else:
        hist, hist_t = [], {"wall_seconds": 0.0, "device_seconds": 0.0}
    mid = getattr(backend, "snapshot", lambda: None)()
    tree0 = _tree_snapshot(backend)
    samples, t = measure(lambda: _run(backend, evaluation))
    after = getattr(backend, "snapshot", lambda: None)()
    tokens = sum(len(s.token_ids) for s in samples)
    record = {
        "name": name,
        "cache_build": {"telemetry": hist_t, "main_model": counter_delta(before, mid), "sequences": len(hist),
                        "tokens": sum(len(s.token_ids) for s in hist)},
        "online": {"telemetry": t, "main_model": counter_delta(mid, after),
                   "draft_cache": counter_delta(tree0, _tree_snapshot(backend)), "sequences": len(samples),
                   "output_tokens": tokens, "output_tokens_per_second": tokens / t["device_seconds"]},
    }
    return record, {s.request_id: tuple(s.token_ids) for s in samples}


def agreement(tokens: dict[str, tuple], baseline: dict[str, tuple]) -> dict[str, float]:
    """Share of requests with identical tokens, and of tokens before the first difference."""
    same = [tokens[k] == baseline[k] for k in baseline]
    prefix = []
    for k, b in baseline.items():
        a = tokens[k]
        n = next((j for j, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))
        prefix.append(n / max(1, len(b)))
    return {"identical_requests": float(np.mean(same)), "mean_matching_prefix": float(np.mean(prefix))}


def algorithm_arm(backend, *, name: str, prompts: Sequence[tuple], length: int, block: int, candidates: int,
                  rollouts: int, seed: int, reward: Callable,
                  history: Sequence[Sequence[GenerationRequest]] = ()) -> dict:
    """One algorithm arm; ``history`` (speculative arms) fills the draft tree first, timed on its own."""
    from ..arllm.algorithms.conditional_is import run_conditional_is
    from ..experimental.arllm.smc_forest import run_smc_rollout_forest
    from ..shared.config import SMCForestConfig

    diagnostics: list[dict] = []

    def run_all() -> list[tuple]:
        outs = []
        for i, prompt in enumerate(prompts):
            seeds = SeedStream(SeedStream(seed).derive("infra", "algorithm", name, i))
            if name.startswith("conditional"):
                res = run_conditional_is(backend, prompt, ConditionalISConfig(
                    candidate_count=candidates, rollout_count=rollouts, block_size=block, total_length=length,
                    reward_temperature=0.5), reward, seeds)
                diagnostics.append({"steps": len(res.steps)})
            elif name.startswith("smc"):
                res = run_smc_rollout_forest(backend, prompt, SMCForestConfig(
                    particle_count=candidates, branch_factor=2, rollout_count=rollouts, block_size=block,
                    total_length=length, reward_temperature=0.5, reuse_rollout_forest=name == "smc_reuse"),
                    reward, seeds)
                diagnostics.append({"steps": len(res.steps), "fresh_rollouts": res.fresh_rollouts,
                                    "reused_rollouts": res.reused_rollouts})
            else:
                raise ValueError(f"unknown algorithm arm {name!r}")
            outs.append(tuple(res.token_ids))
        return outs

    hist, hist_t = measure(lambda: _run(backend, history)) if history else ([], {"wall_seconds": 0.0,
                                                                                  "device_seconds": 0.0})
    before, tree0 = getattr(backend, "snapshot", lambda: None)(), _tree_snapshot(backend)
    outs, t = measure(run_all)
    tokens = sum(len(o) for o in outs)
    return {"name": name, "cache_build": {"telemetry": hist_t, "sequences": len(hist),
                                          "tokens": sum(len(s.token_ids) for s in hist)},
            "online": {"telemetry": t, "main_model": counter_delta(before, getattr(backend, "snapshot", lambda: None)()),
                                     "draft_cache": counter_delta(tree0, _tree_snapshot(backend)),
                                     "problems": len(prompts), "output_tokens": tokens,
                                     "output_tokens_per_second": tokens / t["device_seconds"],
                                     "diagnostics": diagnostics}}


def reuse_arms(backend, *, prompt: tuple, length: int, block: int, updates: int, seed: int, reward: Callable,
               verifier_delay: float) -> list[dict]:
    """Standard, prefetched and delayed-acceptance reward MH on one backend and prompt."""
    import hashlib

    from ..arllm.algorithms.mh import run_reward_mh_chain
    from ..arllm.algorithms.mh_acceleration import run_reward_mh_chain_delayed, run_reward_mh_chain_prefetched
    from ..arllm.config import RewardMHConfig

    calls = {"exact": 0}

    def slow(p, y):
        calls["exact"] += 1
        time.sleep(verifier_delay)
        return reward(p, y)

    cfg = RewardMHConfig(total_length=length, block_size=block, reward_temperature=0.5, iterations=updates)
    sampling = SamplingConfig()
    out, standard = [], None
    for name in ("mh_standard", "mh_prefetched", "mh_delayed"):
        calls["exact"] = 0
        seeds = SeedStream(SeedStream(seed).derive("infra", "reuse"))
        if name == "mh_standard":
            res, t = measure(lambda: run_reward_mh_chain(backend, prompt, cfg, sampling, slow, seeds))
            chain = res
        elif name == "mh_prefetched":
            res, t = measure(lambda: run_reward_mh_chain_prefetched(backend, prompt, cfg, sampling, slow, seeds))
            chain = res.chain
        else:
            res, t = measure(lambda: run_reward_mh_chain_delayed(backend, prompt, cfg, sampling, slow, reward, seeds))
            chain = res
        tokens = tuple(chain.token_ids)
        if standard is None:
            standard = tokens
        accepted = sum(bool(getattr(st, "accepted", False)) for st in chain.trace)
        out.append({"name": name, "online": {"telemetry": t, "exact_reward_evaluations": calls["exact"],
                                             "updates": len(chain.trace), "accepted_updates": accepted,
                                             "token_sha256": hashlib.sha256(np.asarray(tokens, np.int64).tobytes())
                                             .hexdigest()[:16],
                                             "identical_to_standard": tokens == standard}})
    return out


def run_benchmark(make_backend: Callable[[ActiveBatchSpeculationConfig | None], Any], *, prompts: Sequence[tuple],
                  section: str = "all", max_new_tokens: int = 64, batch_sizes: Sequence[int] = (4, 2, 1),
                  history_rollouts: int = 2, draft_tokens: int = 8, block_size: int = 16, candidates: int = 3,
                  rollouts: int = 2, seed: int = 20260812, reward_factory: Callable[[Any], Callable] | None = None,
                  release: Callable[[Any], None] = lambda b: None, mh_updates: int = 8,
                  verifier_delay: float = 0.05) -> dict:
    """All arms of the selected sections; ``make_backend(speculation)`` builds a fresh backend per arm."""
    spec = ActiveBatchSpeculationConfig(tiers=(SpeculationTier(max(batch_sizes), draft_tokens),
                                               SpeculationTier(1 << 20, 0)))
    sampling = SamplingConfig()
    seeds = SeedStream(seed)
    report: dict[str, Any] = {"workload": {"prompts": len(prompts), "prompt_tokens": [len(p) for p in prompts],
                                           "max_new_tokens": max_new_tokens, "batch_sizes": list(batch_sizes),
                                           "history_rollouts": history_rollouts, "draft_tokens": draft_tokens,
                                           "seed": seed}}
    hist = history_batches(prompts, count=history_rollouts, length=max_new_tokens, sampling=sampling, seeds=seeds)
    if section in ("decode", "all"):
        evals = evaluation_batches(prompts, batch_sizes=batch_sizes, length=max_new_tokens, sampling=sampling,
                                   seeds=seeds)
        arms, tokens = [], {}
        for name, s in (("plain", None), ("rollout_tree", spec)):
            b = make_backend(s)
            try:
                rec, tokens[name] = decode_arm(b, name=name, speculative=s is not None, history=hist, evaluation=evals)
            finally:
                release(b)
            arms.append(rec)
        for rec in arms:
            rec["online"]["agreement_with_plain"] = agreement(tokens[rec["name"]], tokens["plain"])
        report["decode"] = arms
    if section in ("algorithm", "all"):
        arms = []
        for name, s in (("conditional_plain", None), ("conditional_rollout_tree", spec), ("smc_no_reuse", None),
                        ("smc_reuse", None)):
            b = make_backend(s)
            try:
                reward = reward_factory(b) if reward_factory is not None else (lambda _p, y: 0.0)
                arms.append(algorithm_arm(b, name=name, prompts=prompts, length=max_new_tokens, block=block_size,
                                          candidates=candidates, rollouts=rollouts, seed=seed, reward=reward,
                                          history=hist if s is not None else ()))
            finally:
                release(b)
        report["algorithm"] = arms
    if section in ("reuse", "all"):
        b = make_backend(None)
        try:
            reward = reward_factory(b) if reward_factory is not None else (lambda _p, y: 0.0)
            report["reuse"] = reuse_arms(b, prompt=tuple(prompts[0]), length=max_new_tokens, block=block_size,
                                         updates=mh_updates, seed=seed, reward=reward, verifier_delay=verifier_delay)
        finally:
            release(b)
        report["workload"].update(mh_updates=mh_updates, verifier_delay_seconds=verifier_delay)
    return report


def _machine() -> dict[str, Any]:
    import torch

    cuda = torch.cuda.is_available()
    return {"platform": platform.platform(), "python": platform.python_version(), "torch": torch.__version__,
            "cuda_runtime": torch.version.cuda, "gpu": torch.cuda.get_device_name(0) if cuda else None}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.rollout_infra")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--model", default="random:qwen2.5-0.5b", help="random:<preset> or a local checkpoint directory")
    p.add_argument("--section", choices=("decode", "algorithm", "reuse", "all"), default="all")
    p.add_argument("--mh-updates", type=int, default=8)
    p.add_argument("--verifier-delay", type=float, default=0.05, help="seconds added to every exact reward")
    p.add_argument("--prompts", type=int, default=2)
    p.add_argument("--prompt-tokens", type=int, default=128)
    p.add_argument("--max-new-tokens", type=int, default=64)
    p.add_argument("--block-size", type=int, default=16)
    p.add_argument("--history-rollouts", type=int, default=2)
    p.add_argument("--batch-sizes", default="4,2,1")
    p.add_argument("--draft-tokens", type=int, default=8)
    p.add_argument("--candidate-count", type=int, default=3)
    p.add_argument("--rollout-count", type=int, default=2)
    p.add_argument("--kv-cache-gb", type=float, default=8.0)
    p.add_argument("--seed", type=int, default=20260812)
    a = p.parse_args(argv)

    from ..arllm.backends.loader import LoadedModel
    from ..arllm.rewards import SequenceLogProbabilityReward

    def make(spec):
        cfg: dict[str, Any] = {"runtime": {"kv_cache_gb": a.kv_cache_gb, "max_batch_size": 64,
                                           "max_sequence_tokens": a.prompt_tokens + a.max_new_tokens + 64}}
        if spec is not None:
            cfg["acceleration"] = {"speculation": {"enabled": True, "stochastic_tree": spec.stochastic_tree,
                                                   "tiers": [[t.max_batch, t.draft_tokens] for t in spec.tiers]}}
        return LoadedModel(a.model, cfg, "base").backend

    def release(b):
        b.close()
        import torch

        torch.cuda.empty_cache()

    if a.model.startswith("random:"):
        from ..models.decoder import PRESETS

        vocab = PRESETS[a.model.split(":", 1)[1]].vocab_size
    else:
        vocab = int(json.loads((Path(a.model) / "config.json").read_text())["vocab_size"])
    rng = np.random.default_rng(a.seed)
    prompts = [tuple(int(t) for t in rng.integers(0, vocab, a.prompt_tokens)) for _ in range(a.prompts)]
    report = run_benchmark(make, prompts=prompts, section=a.section, max_new_tokens=a.max_new_tokens,
                           batch_sizes=[int(x) for x in a.batch_sizes.split(",")],
                           history_rollouts=a.history_rollouts, draft_tokens=a.draft_tokens,
                           block_size=a.block_size, candidates=a.candidate_count, rollouts=a.rollout_count,
                           seed=a.seed, release=release, mh_updates=a.mh_updates, verifier_delay=a.verifier_delay,
                           reward_factory=lambda b: SequenceLogProbabilityReward(b, coefficient=0.5))
    report.update(model=a.model, machine=_machine(), data="synthetic uniform-random prompts, random-init weights"
                  if a.model.startswith("random:") else "synthetic uniform-random prompts")
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(report, indent=2))
    summary = {arm["name"]: round(arm["online"]["output_tokens_per_second"], 1)
               for sec in ("decode", "algorithm") for arm in report.get(sec, [])}
    summary.update({arm["name"]: round(arm["online"]["telemetry"]["wall_seconds"], 2) for arm in report.get("reuse", [])})
    print(json.dumps({"output": str(a.output), "tokens_per_second": summary}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
