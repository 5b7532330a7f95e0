"""Defensive candidate proposals with variance-cost replay allocation for dLLMs.

Reference behaviour: src/inference_scaling/dllm/dynamic_is.py:104-547.  Three
paired arms:

* ``base_candidate_fixed``: candidates from the target policy, a fixed number
  of fresh rollouts each;
* ``trajectory_replay_aware_fixed``: candidates from the defensive mixture
  (1 - a) p_target + a p_aux (outer ratio p_target / mixture, both densities
  exact), history rollouts from the auxiliary model replayed with truncated
  IS plus a fixed fresh tail;
* ``trajectory_replay_aware_optimal``: as above, but history / fresh counts
  come from the variance-cost allocator fed by independent design rollouts
  (design data never enters the estimate).
"""

from __future__ import annotations

from dataclasses import dataclass
from math import exp, isfinite, log
from typing import Literal, Sequence

import numpy as np

from ..shared.budget import BudgetAllocation, VarianceCostEstimate, allocate_variance_cost_budget
from ..shared.rng import SeedStream
from ..shared.types import TokenSequence
from .config import DiffusionISConfig, DiffusionSamplingConfig, diffusion_decision_stage_lengths
from .replay import (DiffusionReplayHistory, DiffusionReplayRewardBatch, DiffusionReplaySelection,
                     build_diffusion_replay_history, select_diffusion_candidates_with_replay)
from .types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample, DiffusionTrajectoryScoreRequest

DynamicDiffusionArm = Literal["base_candidate_fixed", "trajectory_replay_aware_fixed",
                              "trajectory_replay_aware_optimal"]
_ARMS = ("base_candidate_fixed", "trajectory_replay_aware_fixed", "trajectory_replay_aware_optimal")


@dataclass(frozen=True, slots=True)
class DynamicDiffusionDraw:
    sample: DiffusionSample
    source: str
    target_logprob: float
    auxiliary_logprob: float
    mixture_logprob: float
    outer_log_ratio: float


@dataclass(frozen=True, slots=True)
class DynamicDiffusionStep:
    generated_length_before: int
    draws: tuple[DynamicDiffusionDraw, ...]
    allocations: tuple[BudgetAllocation, ...]
    selection: DiffusionReplaySelection
    design_rollouts: int
    evaluation_history_rollouts: int


@dataclass(frozen=True, slots=True)
class DynamicDiffusionResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    arm: DynamicDiffusionArm
    steps: tuple[DynamicDiffusionStep, ...]

    @property
    def rollout_reuse_rate(self) -> float:
        h = sum(c.estimate.history_count for s in self.steps for c in s.selection.candidates)
        f = sum(c.estimate.fresh_count for s in self.steps for c in s.selection.candidates)
        return h / (h + f) if h + f else 0.0


def _score(backend, samples, idx, sampling) -> dict[int, float]:
    if not idx:
        return {}
    got = backend.score_trajectories([DiffusionTrajectoryScoreRequest(samples[i], sampling) for i in idx])
    if len(got) != len(idx):
        raise RuntimeError("backend returned an invalid candidate score count")
    return {i: float(v) for i, v in zip(idx, got)}


def draw_defensive_diffusion_candidates(*, target_backend: DiffusionBackend, auxiliary_backend: DiffusionBackend,
                                        prefix: TokenSequence, generation_length: int, count: int,
                                        sampling: DiffusionSamplingConfig, auxiliary_probability: float, seed: int,
                                        stage_index: int) -> tuple[DynamicDiffusionDraw, ...]:
    """Candidates from the base / auxiliary mixture with the exact outer ratio p_target / mixture."""
    a = auxiliary_probability
    if count <= 0 or not 0 < a < 1:
        raise ValueError("count must be positive and mixture probability must lie in (0, 1)")
    if not sampling.has_exact_trajectory_density:
        raise ValueError("dynamic dLLM candidates require an exact trajectory policy")
    seeds = SeedStream(seed)
    aux = [bool(v) for v in seeds.generator("dllm-dynamic", stage_index, "sources").random(count) < a]
    reqs = [DiffusionGenerationRequest(prefix, generation_length, sampling,
                                       seeds.derive("dllm-dynamic", stage_index, "candidate", c),
                                       f"dllm-dynamic:{stage_index}:candidate:{c}") for c in range(count)]
    t_idx = [i for i in range(count) if not aux[i]]
    a_idx = [i for i in range(count) if aux[i]]
    samples: list[DiffusionSample | None] = [None] * count
    for idx, got in ((t_idx, target_backend.sample_batch([reqs[i] for i in t_idx])),
                     (a_idx, auxiliary_backend.sample_batch([reqs[i] for i in a_idx]))):
        if len(idx) != len(got):
            raise RuntimeError("backend returned an invalid dynamic candidate count")
        for i, s in zip(idx, got):
            if s.trajectory_logprob is None:
                raise RuntimeError("dynamic proposal omitted its trajectory probability")
            samples[i] = s
    tgt = {i: float(samples[i].trajectory_logprob) for i in t_idx}
    tgt.update(_score(target_backend, samples, a_idx, sampling))
    auxs = {i: float(samples[i].trajectory_logprob) for i in a_idx}
    auxs.update(_score(auxiliary_backend, samples, t_idx, sampling))
    out = []
    for i, s in enumerate(samples):
        mix = float(np.logaddexp(log(1 - a) + tgt[i], log(a) + auxs[i]))
        out.append(DynamicDiffusionDraw(s, "auxiliary" if aux[i] else "target", tgt[i], auxs[i], mix, tgt[i] - mix))
    return tuple(out)


def _target_candidates(backend, prefix, length, count, sampling, seed, stage) -> tuple[DynamicDiffusionDraw, ...]:
    seeds = SeedStream(seed)
    got = backend.sample_batch([DiffusionGenerationRequest(prefix, length, sampling,
                                                           seeds.derive("dllm-dynamic-base", stage, c),
                                                           f"dllm-dynamic-base:{stage}:{c}") for c in range(count)])
    if len(got) != count:
        raise RuntimeError("backend returned an invalid base candidate count")
    out = []
    for s in got:
        lp = float(s.trajectory_logprob) if s.trajectory_logprob is not None else 0.0
        out.append(DynamicDiffusionDraw(s, "target", lp, lp, lp, 0.0))
    return tuple(out)


def _std(values: Sequence[float]) -> float:
    if len(values) < 2:
        return 1.0
    v = float(np.std(np.asarray(values, dtype=np.float64), ddof=1))
    return v if isfinite(v) and v >= 0 else 1.0


def _design_statistics(histories, fresh_histories, *, tau: float, truncation: float, history_cost: float,
                       fresh_cost: float) -> tuple[VarianceCostEstimate, ...]:
    if len(histories) != len(fresh_histories):
        raise ValueError("history and fresh design samples must align by candidate")
    lc = log(truncation)
    shift = max((r.reward / tau for d in (*histories, *fresh_histories) for r in d.records), default=0.0)
    out = []
    for h, f in zip(histories, fresh_histories):
        hv = [exp(min(lc, r.target_trajectory_logprob - r.behavior_trajectory_logprob) + r.reward / tau - shift)
              for r in h.records]
        fv = [max(0.0, 1.0 - exp(min(0.0, lc + r.target_trajectory_logprob - r.behavior_trajectory_logprob)))
              * exp(r.reward / tau - shift) for r in f.records]
        out.append(VarianceCostEstimate(_std(hv), _std(fv), history_cost, fresh_cost))
    return tuple(out)


def run_dynamic_diffusion_is(*, arm: DynamicDiffusionArm, target_backend: DiffusionBackend,
                             auxiliary_backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                             sampling: DiffusionSamplingConfig, reward_batch: DiffusionReplayRewardBatch,
                             history_rollouts: int, fresh_rollouts: int, truncation: float,
                             auxiliary_probability: float = 0.5, history_cost: float = 0.05, fresh_cost: float = 1.0,
                             design_rollouts: int = 2, seed: int = 0) -> DynamicDiffusionResult:
    if arm not in _ARMS:
        raise ValueError(f"unknown dynamic dLLM arm {arm!r}")
    for name, v in (("history_rollouts", history_rollouts), ("fresh_rollouts", fresh_rollouts),
                    ("design_rollouts", design_rollouts)):
        if v <= 0:
            raise ValueError(f"{name} must be positive")
    if history_cost <= 0 or fresh_cost <= 0:
        raise ValueError("rollout costs must be positive")
    stages = diffusion_decision_stage_lengths(prompt_length=len(prompt), total_length=config.total_length,
                                              decision_block_size=config.block_size, sampling=sampling)
    seeds = SeedStream(seed)
    generated: TokenSequence = ()
    steps = []
    for si, n in enumerate(stages):
        pre = prompt + generated
        cseed = seeds.derive("dynamic", arm, "candidates")
        draws = (_target_candidates(target_backend, pre, n, config.candidate_count, sampling, cseed, si)
                 if arm == "base_candidate_fixed" else
                 draw_defensive_diffusion_candidates(target_backend=target_backend,
                                                     auxiliary_backend=auxiliary_backend, prefix=pre,
                                                     generation_length=n, count=config.candidate_count,
                                                     sampling=sampling, auxiliary_probability=auxiliary_probability,
                                                     seed=cseed, stage_index=si))
        cands = tuple(d.sample for d in draws)
        rest = config.total_length - len(generated) - n
        hist: tuple[DiffusionReplayHistory, ...] | None = None
        design = evaluation = 0
        common = dict(prompt=prompt, generated_prefix=generated, candidates=cands, rollout_length=rest,
                      target_sampling=sampling, behavior_sampling=sampling, reward_batch=reward_batch)
        if rest == 0:
            fresh = (1,) * len(cands)
            allocs = tuple(BudgetAllocation(0, 0, 0.0, 0.0, 0.0) for _ in cands)
        elif arm == "base_candidate_fixed":
            fresh = (history_rollouts + fresh_rollouts,) * len(cands)
            allocs = tuple(BudgetAllocation(0, c, 0.0, float(c), float(c)) for c in fresh)
        else:
            hist = build_diffusion_replay_history(target_backend=target_backend, behavior_backend=auxiliary_backend,
                                                  count_per_candidate=history_rollouts,
                                                  seed=seeds.derive("dynamic", arm, "evaluation-history", si),
                                                  **common)
            evaluation = sum(len(h.records) for h in hist)
            if arm == "trajectory_replay_aware_fixed":
                fresh = (fresh_rollouts,) * len(cands)
                allocs = tuple(BudgetAllocation(len(h.records), fresh_rollouts, float(len(h.records)),
                                                float(fresh_rollouts),
                                                len(h.records) * history_cost + fresh_rollouts * fresh_cost)
                               for h in hist)
            else:
                d_hist = build_diffusion_replay_history(target_backend=target_backend,
                                                        behavior_backend=auxiliary_backend,
                                                        count_per_candidate=design_rollouts,
                                                        seed=seeds.derive("dynamic", arm, "design-history", si),
                                                        **common)
                # an independent target-policy pilot; swapping the roles yields both exact densities
                d_fresh = build_diffusion_replay_history(target_backend=auxiliary_backend,
                                                         behavior_backend=target_backend,
                                                         count_per_candidate=design_rollouts,
                                                         seed=seeds.derive("dynamic", arm, "design-fresh", si),
                                                         **common)
                design = sum(len(h.records) for hs in (d_hist, d_fresh) for h in hs)
                stats = _design_statistics(d_hist, d_fresh, tau=config.reward_temperature, truncation=truncation,
                                           history_cost=history_cost, fresh_cost=fresh_cost)
                groups = tuple(h.rollout_prefix for h in hist)
                caps = tuple(len(h.records) for h in hist)
                gcap: dict = {}
                for g, c in zip(groups, caps):
                    gcap[g] = gcap.get(g, 0) + c
                allocs = allocate_variance_cost_budget(
                    outer_ratios=[exp(d.outer_log_ratio) for d in draws], statistics=stats,
                    history_capacities=caps, history_groups=groups, group_capacities=gcap,
                    rollout_budget=len(cands) * (history_rollouts * history_cost + fresh_rollouts * fresh_cost),
                    minimum_fresh=1)
                hist = tuple(DiffusionReplayHistory(h.rollout_prefix, h.records[:a.history_count])
                             for h, a in zip(hist, allocs))
                fresh = tuple(a.fresh_count for a in allocs)
        sel = select_diffusion_candidates_with_replay(
            target_backend=target_backend, behavior_backend=auxiliary_backend if hist is not None else None,
            prompt=prompt, generated_prefix=generated, candidates=cands, histories=hist, rollout_length=rest,
            fresh_count=fresh, target_sampling=sampling, behavior_sampling=sampling if hist is not None else None,
            reward_batch=reward_batch, reward_temperature=config.reward_temperature, truncation=truncation,
            seed=seeds.derive("dynamic", arm, "selection", si), candidate_log_ratios=[d.outer_log_ratio for d in draws])
        steps.append(DynamicDiffusionStep(len(generated), draws, allocs, sel, design, evaluation))
        generated += sel.selected.sample.token_ids
    return DynamicDiffusionResult(prompt, generated, arm, tuple(steps))


__all__ = ["DynamicDiffusionArm", "DynamicDiffusionDraw", "DynamicDiffusionResult", "DynamicDiffusionStep",
           "draw_defensive_diffusion_candidates", "run_dynamic_diffusion_is"]
