"""Defensive candidate proposals with variance-cost replay allocation for dLLMs.

Three paired arms, each a small strategy object that decides, per decision block,
which rollouts weight the candidates:

* ``base_candidate_fixed``: candidates from the target policy and a fixed number of
  fresh rollouts each;
* ``trajectory_replay_aware_fixed``: candidates from the defensive mixture
  (1 - a) p_target + a p_aux (outer ratio p_target / mixture, both densities exact);
  auxiliary-model history rollouts replayed with truncated IS plus a fixed fresh tail;
* ``trajectory_replay_aware_optimal``: as above, with history / fresh counts from the
  variance-cost allocator, fed by independent design rollouts that never enter the
  estimate.

Arm names, stream names and request ids follow src/inference_scaling/dllm/dynamic_is.py.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import log
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


def _trajectory_scores(backend, samples: Sequence[DiffusionSample], sampling) -> np.ndarray:
    if not samples:
        return np.zeros(0)
    got = backend.score_trajectories([DiffusionTrajectoryScoreRequest(s, sampling) for s in samples])
    if len(got) != len(samples):
        raise RuntimeError(f"{len(got)} trajectory scores for {len(samples)} candidates")
    return np.asarray([float(v) for v in got])


def draw_defensive_diffusion_candidates(*, target_backend: DiffusionBackend, auxiliary_backend: DiffusionBackend,
                                        prefix: TokenSequence, generation_length: int, count: int,
                                        sampling: DiffusionSamplingConfig, auxiliary_probability: float, seed: int,
                                        stage_index: int) -> tuple[DynamicDiffusionDraw, ...]:
    """Candidates from the target / auxiliary mixture with the exact outer ratio p_target / mixture."""
    a = auxiliary_probability
    if count < 1 or not 0.0 < a < 1.0:
        raise ValueError("count must be positive and the mixture probability must lie in (0, 1)")
    if not sampling.has_exact_trajectory_density:
        raise ValueError("defensive candidates need a policy with exact trajectory densities")
    seeds = SeedStream(seed)
    from_aux = seeds.generator("dllm-dynamic", stage_index, "sources").random(count) < a
    requests = [DiffusionGenerationRequest(prefix, generation_length, sampling,
                                           seeds.derive("dllm-dynamic", stage_index, "candidate", c),
                                           f"dllm-dynamic:{stage_index}:candidate:{c}") for c in range(count)]
    samples: list = [None] * count
    for backend, mask in ((target_backend, ~from_aux), (auxiliary_backend, from_aux)):
        rows = np.flatnonzero(mask)
        got = backend.sample_batch([requests[i] for i in rows])
        if len(got) != rows.size:
            raise RuntimeError(f"{len(got)} candidates for {rows.size} requests")
        for i, sample in zip(rows, got):
            if sample.trajectory_logprob is None:
                raise RuntimeError("a defensive candidate came without its trajectory probability")
            samples[i] = sample
    own = np.asarray([float(s.trajectory_logprob) for s in samples])
    target = own.copy()
    auxiliary = own.copy()
    # each sample's density under the policy that did NOT draw it needs one scoring pass
    target[from_aux] = _trajectory_scores(target_backend, [samples[i] for i in np.flatnonzero(from_aux)], sampling)
    auxiliary[~from_aux] = _trajectory_scores(auxiliary_backend, [samples[i] for i in np.flatnonzero(~from_aux)],
                                              sampling)
    mixture = np.logaddexp(log(1.0 - a) + target, log(a) + auxiliary)
    return tuple(DynamicDiffusionDraw(s, "auxiliary" if aux else "target", float(t), float(x), float(m), float(t - m))
                 for s, aux, t, x, m in zip(samples, from_aux, target, auxiliary, mixture))


def _target_candidates(backend, prefix, length, count, sampling, seed, stage) -> tuple[DynamicDiffusionDraw, ...]:
    seeds = SeedStream(seed)
    requests = [DiffusionGenerationRequest(prefix, length, sampling, seeds.derive("dllm-dynamic-base", stage, c),
                                           f"dllm-dynamic-base:{stage}:{c}") for c in range(count)]
    got = backend.sample_batch(requests)
    if len(got) != count:
        raise RuntimeError(f"{len(got)} base candidates for {count}")
    draws = []
    for s in got:
        lp = 0.0 if s.trajectory_logprob is None else float(s.trajectory_logprob)
        draws.append(DynamicDiffusionDraw(s, "target", lp, lp, lp, 0.0))
    return tuple(draws)


def _sample_std(values: np.ndarray) -> float:
    if values.size < 2:
        return 1.0
    spread = float(values.std(ddof=1))
    return spread if np.isfinite(spread) and spread >= 0 else 1.0


def _design_statistics(histories, fresh_histories, *, tau: float, truncation: float, history_cost: float,
                       fresh_cost: float) -> tuple[VarianceCostEstimate, ...]:
    """Per-candidate spread of the history and fresh-tail terms, from design rollouts only."""
    if len(histories) != len(fresh_histories):
        raise ValueError("design histories and fresh designs must pair up by candidate")
    log_c = log(truncation)

    def columns(records):
        arr = np.asarray([(r.target_trajectory_logprob - r.behavior_trajectory_logprob, r.reward / tau)
                          for r in records], dtype=np.float64).reshape(-1, 2)
        return arr[:, 0], arr[:, 1]

    everything = [r.reward / tau for group in (*histories, *fresh_histories) for r in group.records]
    shift = max(everything, default=0.0)
    stats = []
    for h, f in zip(histories, fresh_histories):
        ratio_h, scaled_h = columns(h.records)
        ratio_f, scaled_f = columns(f.records)
        history_terms = np.exp(np.minimum(log_c, ratio_h) + scaled_h - shift)
        tail = np.maximum(0.0, 1.0 - np.exp(np.minimum(0.0, log_c + ratio_f)))
        fresh_terms = tail * np.exp(scaled_f - shift)
        stats.append(VarianceCostEstimate(_sample_std(history_terms), _sample_std(fresh_terms), history_cost,
                                          fresh_cost))
    return tuple(stats)


@dataclass
class _StagePlan:
    histories: tuple[DiffusionReplayHistory, ...] | None
    fresh: tuple[int, ...]
    allocations: tuple[BudgetAllocation, ...]
    design: int = 0
    evaluation: int = 0


class _DynamicRun:
    def __init__(self, arm, target_backend, auxiliary_backend, prompt, config, sampling, reward_batch,
                 history_rollouts, fresh_rollouts, truncation, auxiliary_probability, history_cost, fresh_cost,
                 design_rollouts, seeds):
        self.arm = arm
        self.target = target_backend
        self.auxiliary = auxiliary_backend
        self.prompt = tuple(prompt)
        self.config = config
        self.sampling = sampling
        self.reward_batch = reward_batch
        self.history_rollouts = history_rollouts
        self.fresh_rollouts = fresh_rollouts
        self.truncation = truncation
        self.a = auxiliary_probability
        self.history_cost = history_cost
        self.fresh_cost = fresh_cost
        self.design_rollouts = design_rollouts
        self.seeds = seeds

    def draws(self, generated, length, stage):
        seed = self.seeds.derive("dynamic", self.arm, "candidates")
        prefix = self.prompt + tuple(generated)
        if self.arm == "base_candidate_fixed":
            return _target_candidates(self.target, prefix, length, self.config.candidate_count, self.sampling, seed,
                                      stage)
        return draw_defensive_diffusion_candidates(
            target_backend=self.target, auxiliary_backend=self.auxiliary, prefix=prefix, generation_length=length,
            count=self.config.candidate_count, sampling=self.sampling, auxiliary_probability=self.a, seed=seed,
            stage_index=stage)

    def _history(self, generated, candidates, remaining, count, name, stage, *, swap=False):
        target, behaviour = (self.auxiliary, self.target) if swap else (self.target, self.auxiliary)
        return build_diffusion_replay_history(
            target_backend=target, behavior_backend=behaviour, prompt=self.prompt, generated_prefix=generated,
            candidates=candidates, rollout_length=remaining, count_per_candidate=count,
            target_sampling=self.sampling, behavior_sampling=self.sampling, reward_batch=self.reward_batch,
            seed=self.seeds.derive("dynamic", self.arm, name, stage))

    def plan(self, generated, candidates, draws, remaining, stage) -> _StagePlan:
        n = len(candidates)
        if remaining == 0:
            return _StagePlan(None, (1,) * n, tuple(BudgetAllocation(0, 0, 0.0, 0.0, 0.0) for _ in candidates))
        if self.arm == "base_candidate_fixed":
            total = self.history_rollouts + self.fresh_rollouts
            return _StagePlan(None, (total,) * n,
                              tuple(BudgetAllocation(0, total, 0.0, float(total), float(total)) for _ in candidates))
        histories = self._history(generated, candidates, remaining, self.history_rollouts, "evaluation-history",
                                  stage)
        evaluation = sum(len(h.records) for h in histories)
        if self.arm == "trajectory_replay_aware_fixed":
            f = self.fresh_rollouts
            allocations = tuple(BudgetAllocation(len(h.records), f, float(len(h.records)), float(f),
                                                 len(h.records) * self.history_cost + f * self.fresh_cost)
                                for h in histories)
            return _StagePlan(histories, (f,) * n, allocations, 0, evaluation)
        design_h = self._history(generated, candidates, remaining, self.design_rollouts, "design-history", stage)
        # an independent target-policy pilot: with the roles swapped both exact densities come out
        design_f = self._history(generated, candidates, remaining, self.design_rollouts, "design-fresh", stage,
                                 swap=True)
        design = sum(len(h.records) for group in (design_h, design_f) for h in group)
        stats = _design_statistics(design_h, design_f, tau=self.config.reward_temperature, truncation=self.truncation,
                                   history_cost=self.history_cost, fresh_cost=self.fresh_cost)
        groups = tuple(h.rollout_prefix for h in histories)
        capacities = tuple(len(h.records) for h in histories)
        group_caps: dict = {}
        for g, c in zip(groups, capacities):
            group_caps[g] = group_caps.get(g, 0) + c
        budget = n * (self.history_rollouts * self.history_cost + self.fresh_rollouts * self.fresh_cost)
        allocations = allocate_variance_cost_budget(
            outer_ratios=np.exp([d.outer_log_ratio for d in draws]).tolist(), statistics=stats,
            history_capacities=capacities, history_groups=groups, group_capacities=group_caps,
            rollout_budget=budget, minimum_fresh=1)
        trimmed = tuple(DiffusionReplayHistory(h.rollout_prefix, h.records[:a.history_count])
                        for h, a in zip(histories, allocations))
        return _StagePlan(trimmed, tuple(a.fresh_count for a in allocations), allocations, design, evaluation)


def run_dynamic_diffusion_is(*, arm: DynamicDiffusionArm, target_backend: DiffusionBackend,
                             auxiliary_backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                             sampling: DiffusionSamplingConfig, reward_batch: DiffusionReplayRewardBatch,
                             history_rollouts: int, fresh_rollouts: int, truncation: float,
                             auxiliary_probability: float = 0.5, history_cost: float = 0.05, fresh_cost: float = 1.0,
                             design_rollouts: int = 2, seed: int = 0) -> DynamicDiffusionResult:
    if arm not in _ARMS:
        raise ValueError(f"arm {arm!r} is not one of {_ARMS}")
    counts = {"history_rollouts": history_rollouts, "fresh_rollouts": fresh_rollouts,
              "design_rollouts": design_rollouts}
    bad = [name for name, value in counts.items() if value < 1]
    if bad:
        raise ValueError(f"{', '.join(bad)} must be positive")
    if not (history_cost > 0 and fresh_cost > 0):
        raise ValueError("rollout costs have to be positive")
    stages = diffusion_decision_stage_lengths(prompt_length=len(prompt), total_length=config.total_length,
                                              decision_block_size=config.block_size, sampling=sampling)
    seeds = SeedStream(seed)
    run = _DynamicRun(arm, target_backend, auxiliary_backend, prompt, config, sampling, reward_batch,
                      history_rollouts, fresh_rollouts, truncation, auxiliary_probability, history_cost, fresh_cost,
                      design_rollouts, seeds)
    generated: tuple = ()
    steps = []
    for stage, length in enumerate(stages):
        draws = run.draws(generated, length, stage)
        candidates = tuple(d.sample for d in draws)
        remaining = config.total_length - len(generated) - length
        plan = run.plan(generated, candidates, draws, remaining, stage)
        replaying = plan.histories is not None
        selection = select_diffusion_candidates_with_replay(
            target_backend=target_backend, behavior_backend=auxiliary_backend if replaying else None,
            prompt=prompt, generated_prefix=generated, candidates=candidates, histories=plan.histories,
            rollout_length=remaining, fresh_count=plan.fresh, target_sampling=sampling,
            behavior_sampling=sampling if replaying else None, reward_batch=reward_batch,
            reward_temperature=config.reward_temperature, truncation=truncation,
            seed=seeds.derive("dynamic", arm, "selection", stage),
            candidate_log_ratios=[d.outer_log_ratio for d in draws])
        steps.append(DynamicDiffusionStep(len(generated), draws, plan.allocations, selection, plan.design,
                                          plan.evaluation))
        generated += tuple(selection.selected.sample.token_ids)
    return DynamicDiffusionResult(tuple(prompt), generated, arm, tuple(steps))


__all__ = ["DynamicDiffusionArm", "DynamicDiffusionDraw", "DynamicDiffusionResult", "DynamicDiffusionStep",
           "draw_defensive_diffusion_candidates", "run_dynamic_diffusion_is"]
