"""Adaptive rollout allocation for diffusion conditional IS, with pilots kept apart.

Per decision block: draw candidates; run independent pilot rollouts to estimate each
candidate's standard deviation of exp(r / tau) (all shifted by the common maximum);
freeze a fresh-rollout allocation with the variance-cost allocator; then weight and
select using fresh evaluation rollouts only.  Pilot draws never enter the estimate, so
it stays unbiased.  Stream names and request ids follow
src/inference_scaling/dllm/algorithms/progressive_is.py.
"""

from __future__ import annotations

from dataclasses import dataclass
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
    """Sample standard deviation of exp(r / tau - shift) over each candidate's pilot rollouts."""
    k = len(candidates)
    requests = [DiffusionGenerationRequest(tuple(prompt) + tuple(generated) + tuple(candidates[c].token_ids), length,
                                           sampling, seeds.derive("dllm-progressive", step, "pilot", c, r),
                                           f"dllm-progressive:{step}:candidate:{c}:pilot:{r}")
                for c in range(k) for r in range(count)]
    pilots = backend.sample_batch(requests)
    if len(pilots) != len(requests):
        raise RuntimeError(f"{len(pilots)} pilot rollouts came back for {len(requests)}")
    texts = [tuple(generated) + tuple(candidates[i // count].token_ids) + tuple(s.token_ids)
             for i, s in enumerate(pilots)]
    scaled = np.asarray([float(v) for v in reward_batch(prompt, texts)], dtype=np.float64) / tau
    if scaled.shape != (len(pilots),) or not np.isfinite(scaled).all():
        raise RuntimeError("the reward batch returned missing or non-finite pilot rewards")
    tilted = np.exp(scaled.reshape(k, count) - scaled.max())
    if count < 2:
        return (1.0,) * k
    spread = tilted.std(axis=1, ddof=1)
    return tuple(np.where(np.isfinite(spread) & (spread >= 0), spread, 1.0).tolist())


def _candidates(backend, prompt, generated, length, sampling, seeds, step, count) -> tuple[DiffusionSample, ...]:
    requests = [DiffusionGenerationRequest(tuple(prompt) + tuple(generated), length, sampling,
                                           seeds.derive("dllm-progressive", step, "candidate", c),
                                           f"dllm-progressive:{step}:candidate:{c}") for c in range(count)]
    drawn = tuple(backend.sample_batch(requests))
    if len(drawn) != count:
        raise RuntimeError(f"{len(drawn)} candidates came back for {count}")
    return drawn


def run_progressive_diffusion_is(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                                 sampling: DiffusionSamplingConfig, reward_batch: DiffusionReplayRewardBatch,
                                 pilot_rollouts_per_candidate: int, evaluation_rollout_budget: int, seed: int = 0
                                 ) -> ProgressiveDiffusionISResult:
    if pilot_rollouts_per_candidate < 1:
        raise ValueError("pilot_rollouts_per_candidate has to be positive")
    if evaluation_rollout_budget < config.candidate_count:
        raise ValueError("the evaluation budget must give every candidate at least one rollout")
    stages = diffusion_decision_stage_lengths(prompt_length=len(prompt), total_length=config.total_length,
                                              decision_block_size=config.block_size, sampling=sampling)
    seeds = SeedStream(seed)
    generated: tuple = ()
    steps = []
    for step, length in enumerate(stages):
        cands = _candidates(backend, prompt, generated, length, sampling, seeds, step, config.candidate_count)
        remaining = config.total_length - len(generated) - length
        if remaining == 0:
            allocations = tuple(BudgetAllocation(0, 0, 0.0, 0.0, 0.0) for _ in cands)
            fresh, pilots = (1,) * len(cands), 0
        else:
            deviations = _pilot_deviations(backend, prompt, generated, cands, remaining, pilot_rollouts_per_candidate,
                                           sampling, reward_batch, config.reward_temperature, seeds, step)
            pilots = len(cands) * pilot_rollouts_per_candidate
            ones = (1.0,) * len(cands)
            allocations = allocate_fresh_rollout_budget(outer_ratios=ones, standard_deviations=deviations, costs=ones,
                                                        rollout_budget=float(evaluation_rollout_budget),
                                                        minimum_fresh=1)
            fresh = tuple(a.fresh_count for a in allocations)
        selection = select_diffusion_candidates_with_replay(
            target_backend=backend, behavior_backend=None, prompt=prompt, generated_prefix=generated, candidates=cands,
            histories=None, rollout_length=remaining, fresh_count=fresh, target_sampling=sampling,
            behavior_sampling=None, reward_batch=reward_batch, reward_temperature=config.reward_temperature,
            truncation=1.0, seed=seeds.derive("dllm-progressive", step, "selection"))
        steps.append(ProgressiveDiffusionISStep(len(generated), cands, allocations, pilots, selection))
        generated += tuple(selection.selected.sample.token_ids)
    return ProgressiveDiffusionISResult(prompt, generated, tuple(steps))


__all__ = ["ProgressiveDiffusionISResult", "ProgressiveDiffusionISStep", "run_progressive_diffusion_is"]
