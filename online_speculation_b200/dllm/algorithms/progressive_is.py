"""Pilot / evaluation-separated adaptive rollout allocation for diffusion conditional IS.

Reference behaviour: src/inference_scaling/dllm/algorithms/progressive_is.py:146-245.
Per decision block: draw candidates, run independent pilot rollouts to
estimate each candidate's standard deviation of exp(r / tau) (shifted by the
common maximum for stability), freeze a fresh-rollout allocation from the
variance-cost allocator, then weight and select with fresh evaluation
rollouts only (pilot draws never enter the estimate, so the estimate stays
unbiased).
"""

from __future__ import annotations

from dataclasses import dataclass
from math import exp, isfinite
from typing import Sequence

import numpy as np

from ...shared.budget import BudgetAllocation, allocate_fresh_rollout_budget
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import DiffusionISConfig, DiffusionSamplingConfig, diffusion_decision_stage_lengths
from ..replay import DiffusionReplayRewardBatch, DiffusionReplaySelection, select_diffusion_candidates_with_replay
from ..types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample


@dataclass(frozen=True, slots=True)
class ProgressiveDiffusionISStep:
    generated_length_before: int
    candidates: tuple[DiffusionSample, ...]
    allocations: tuple[BudgetAllocation, ...]
    pilot_rollouts: int
    selection: DiffusionReplaySelection


@dataclass(frozen=True, slots=True)
class ProgressiveDiffusionISResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[ProgressiveDiffusionISStep, ...]


def _pilot_deviations(backend, prompt, generated, candidates: Sequence[DiffusionSample], length: int, count: int,
                      sampling, reward_batch, tau: float, seeds: SeedStream, step: int) -> tuple[float, ...]:
    reqs, owners = [], []
    for ci, c in enumerate(candidates):
        for r in range(count):
            reqs.append(DiffusionGenerationRequest(prompt + generated + c.token_ids, length, sampling,
                                                   seeds.derive("dllm-progressive", step, "pilot", ci, r),
                                                   f"dllm-progressive:{step}:candidate:{ci}:pilot:{r}"))
            owners.append(ci)
    samples = backend.sample_batch(reqs)
    if len(samples) != len(reqs):
        raise RuntimeError("backend returned an invalid progressive pilot count")
    rewards = [float(v) for v in reward_batch(prompt, [generated + candidates[o].token_ids + s.token_ids
                                                       for o, s in zip(owners, samples)])]
    if len(rewards) != len(samples) or not all(isfinite(v) for v in rewards):
        raise RuntimeError("reward evaluator returned an invalid progressive pilot count")
    grouped: list[list[float]] = [[] for _ in candidates]
    for o, r in zip(owners, rewards):
        grouped[o].append(r / tau)
    shift = max((v for g in grouped for v in g), default=0.0)
    out = []
    for g in grouped:
        d = float(np.std([exp(v - shift) for v in g], ddof=1)) if len(g) >= 2 else 1.0
        out.append(d if isfinite(d) and d >= 0 else 1.0)
    return tuple(out)


def run_progressive_diffusion_is(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                                 sampling: DiffusionSamplingConfig, reward_batch: DiffusionReplayRewardBatch,
                                 pilot_rollouts_per_candidate: int, evaluation_rollout_budget: int, seed: int = 0
                                 ) -> ProgressiveDiffusionISResult:
    if pilot_rollouts_per_candidate <= 0:
        raise ValueError("pilot_rollouts_per_candidate must be positive")
    if evaluation_rollout_budget < config.candidate_count:
        raise ValueError("evaluation budget must cover one rollout per candidate")
    stages = diffusion_decision_stage_lengths(prompt_length=len(prompt), total_length=config.total_length,
                                              decision_block_size=config.block_size, sampling=sampling)
    seeds = SeedStream(seed)
    generated: TokenSequence = ()
    steps = []
    for si, n in enumerate(stages):
        cands = tuple(backend.sample_batch([
            DiffusionGenerationRequest(prompt + generated, n, sampling,
                                       seeds.derive("dllm-progressive", si, "candidate", c),
                                       f"dllm-progressive:{si}:candidate:{c}") for c in range(config.candidate_count)]))
        if len(cands) != config.candidate_count:
            raise RuntimeError("backend returned an invalid progressive candidate count")
        rest = config.total_length - len(generated) - n
        if rest == 0:
            allocs = tuple(BudgetAllocation(0, 0, 0.0, 0.0, 0.0) for _ in cands)
            fresh, pilots = (1,) * len(cands), 0
        else:
            devs = _pilot_deviations(backend, prompt, generated, cands, rest, pilot_rollouts_per_candidate, sampling,
                                     reward_batch, config.reward_temperature, seeds, si)
            pilots = len(cands) * pilot_rollouts_per_candidate
            allocs = allocate_fresh_rollout_budget(outer_ratios=(1.0,) * len(cands), standard_deviations=devs,
                                                   costs=(1.0,) * len(cands),
                                                   rollout_budget=float(evaluation_rollout_budget), minimum_fresh=1)
            fresh = tuple(a.fresh_count for a in allocs)
        sel = select_diffusion_candidates_with_replay(
            target_backend=backend, behavior_backend=None, prompt=prompt, generated_prefix=generated, candidates=cands,
            histories=None, rollout_length=rest, fresh_count=fresh, target_sampling=sampling, behavior_sampling=None,
            reward_batch=reward_batch, reward_temperature=config.reward_temperature, truncation=1.0,
            seed=seeds.derive("dllm-progressive", si, "selection"))
        steps.append(ProgressiveDiffusionISStep(len(generated), cands, allocs, pilots, sel))
        generated += sel.selected.sample.token_ids
    return ProgressiveDiffusionISResult(prompt, generated, tuple(steps))


__all__ = ["ProgressiveDiffusionISResult", "ProgressiveDiffusionISStep", "run_progressive_diffusion_is"]
