"""Exact trajectory replay for block-diffusion rollout weights.

History rollouts are drawn once from a behaviour policy and scored under the target
policy.  A candidate's weight combines truncated-IS history terms
min(c, p / q) exp(r / tau) with fresh target rollouts, whose tail correction
(1 - c q / p)+ keeps the estimate unbiased; with exact trajectory densities p / q is
the ratio of the same reverse trace under the two policies.  Rollouts of all
candidates are laid out as one (candidate x rollout) grid per call.  Stream names and
request ids follow src/inference_scaling/dllm/replay.py (frozen histories replay).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import isfinite
from typing import Callable

import numpy as np

from ..shared.importance import ProbabilityObservation, ReplayWeightEstimate, TruncatedReplayRolloutWeightProvider, \
    logmeanexp
from ..shared.rng import SeedStream
from ..shared.stepwise import normalize_log_weights
from ..shared.types import TokenSequence
from .config import DiffusionSamplingConfig
from .types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample, DiffusionTrajectoryScoreRequest

DiffusionReplayRewardBatch = Callable[[TokenSequence, Sequence[TokenSequence]], Sequence[float]]


def validate_exact_pair(target: DiffusionSamplingConfig, behavior: DiffusionSamplingConfig) -> None:
    if not (target.has_exact_trajectory_density and behavior.has_exact_trajectory_density):
        raise ValueError("replay weights need exact trajectory densities under both policies")
    schedule = ("block_length", "steps_per_block", "remasking", "mask_token_id")
    if any(getattr(target, f) != getattr(behavior, f) for f in schedule):
        raise ValueError("target and behaviour trajectories must follow the same schedule")


@dataclass(frozen=True, slots=True)
class DiffusionReplayRecord:
    rollout_prefix: TokenSequence
    sample: DiffusionSample
    target_trajectory_logprob: float
    behavior_trajectory_logprob: float
    reward: float

    def __post_init__(self) -> None:
        if self.sample.prefix != self.rollout_prefix:
            raise ValueError("replay sample prefix does not match its cache key")
        if not (isfinite(self.target_trajectory_logprob) and isfinite(self.behavior_trajectory_logprob)):
            raise ValueError("target and behavior trajectory probabilities must be finite")

    @property
    def observation(self) -> ProbabilityObservation:
        return ProbabilityObservation(self.target_trajectory_logprob, self.behavior_trajectory_logprob, self.reward)


@dataclass(frozen=True, slots=True)
class DiffusionReplayHistory:
    rollout_prefix: TokenSequence
    records: tuple[DiffusionReplayRecord, ...]

    def __post_init__(self) -> None:
        if any(r.rollout_prefix != self.rollout_prefix for r in self.records):
            raise ValueError("replay history mixes different rollout prefixes")


@dataclass(frozen=True, slots=True)
class DiffusionReplayCandidate:
    sample: DiffusionSample
    estimate: ReplayWeightEstimate
    outer_log_ratio: float = 0.0


@dataclass(frozen=True, slots=True)
class DiffusionReplaySelection:
    candidates: tuple[DiffusionReplayCandidate, ...]
    probabilities: tuple[float, ...]
    selected_index: int
    fresh_records: tuple[tuple[DiffusionReplayRecord, ...], ...]

    @property
    def selected(self) -> DiffusionReplayCandidate:
        return self.candidates[self.selected_index]


def _rewards(reward_batch, prompt, texts, what: str) -> list[float]:
    values = [float(v) for v in reward_batch(prompt, texts)]
    if len(values) != len(texts):
        raise RuntimeError(f"{len(values)} {what} rewards for {len(texts)} rollouts")
    return values


def _grid(counts: Sequence[int]) -> list[tuple[int, int]]:
    """(candidate, index) cells of a ragged candidate x rollout grid, row by row."""
    return [(c, i) for c, n in enumerate(counts) for i in range(n)]


def build_diffusion_replay_history(*, target_backend: DiffusionBackend, behavior_backend: DiffusionBackend,
                                   prompt: TokenSequence, generated_prefix: TokenSequence,
                                   candidates: Sequence[DiffusionSample], rollout_length: int,
                                   count_per_candidate: int, target_sampling: DiffusionSamplingConfig,
                                   behavior_sampling: DiffusionSamplingConfig,
                                   reward_batch: DiffusionReplayRewardBatch, seed: int
                                   ) -> tuple[DiffusionReplayHistory, ...]:
    """Draw immutable behaviour trajectories per candidate and score them under the target once."""
    validate_exact_pair(target_sampling, behavior_sampling)
    if count_per_candidate < 1:
        raise ValueError("count_per_candidate has to be positive")
    prefixes = [tuple(prompt) + tuple(generated_prefix) + tuple(c.token_ids) for c in candidates]
    if rollout_length <= 0:
        return tuple(DiffusionReplayHistory(p, ()) for p in prefixes)
    seeds = SeedStream(seed)
    cells = _grid([count_per_candidate] * len(candidates))
    requests = [DiffusionGenerationRequest(prefixes[c], rollout_length, behavior_sampling,
                                           seeds.derive("dllm-replay", c, h), f"dllm-replay:{c}:{h}") for c, h in cells]
    drawn = behavior_backend.sample_batch(requests)
    if len(drawn) != len(requests):
        raise RuntimeError(f"{len(drawn)} behaviour rollouts for {len(requests)} requests")
    if any(s.trajectory_logprob is None for s in drawn):
        raise RuntimeError("a behaviour rollout came without its trajectory probability")
    target = target_backend.score_trajectories([DiffusionTrajectoryScoreRequest(s, target_sampling) for s in drawn])
    if len(target) != len(drawn):
        raise RuntimeError(f"{len(target)} target scores for {len(drawn)} rollouts")
    texts = [tuple(generated_prefix) + tuple(candidates[c].token_ids) + tuple(s.token_ids)
             for (c, _), s in zip(cells, drawn)]
    rewards = _rewards(reward_batch, prompt, texts, "replay")
    rows: list[list[DiffusionReplayRecord]] = [[] for _ in candidates]
    for (c, _), s, t, r in zip(cells, drawn, target, rewards):
        rows[c].append(DiffusionReplayRecord(s.prefix, s, float(t), float(s.trajectory_logprob), r))
    return tuple(DiffusionReplayHistory(p, tuple(row)) for p, row in zip(prefixes, rows))


def _terminal_selection(candidates, outer, rewards, tau, seed) -> DiffusionReplaySelection:
    chosen = tuple(DiffusionReplayCandidate(c, ReplayWeightEstimate(r / tau, (), (r / tau,)), o)
                   for c, r, o in zip(candidates, rewards, outer))
    probabilities = normalize_log_weights([c.estimate.log_weight + c.outer_log_ratio for c in chosen])
    pick = int(np.random.default_rng(seed).choice(len(chosen), p=probabilities))
    return DiffusionReplaySelection(chosen, probabilities, pick, tuple(() for _ in candidates))


def select_diffusion_candidates_with_replay(*, target_backend: DiffusionBackend,
                                            behavior_backend: DiffusionBackend | None, prompt: TokenSequence,
                                            generated_prefix: TokenSequence, candidates: Sequence[DiffusionSample],
                                            histories: Sequence[DiffusionReplayHistory] | None, rollout_length: int,
                                            fresh_count: int | Sequence[int],
                                            target_sampling: DiffusionSamplingConfig,
                                            behavior_sampling: DiffusionSamplingConfig | None,
                                            reward_batch: DiffusionReplayRewardBatch, reward_temperature: float,
                                            truncation: float, seed: int,
                                            candidate_log_ratios: Sequence[float] | None = None
                                            ) -> DiffusionReplaySelection:
    """Weight each candidate from fresh rollouts, or corrected replay plus a fresh tail, then draw one."""
    n = len(candidates)
    if n == 0:
        raise ValueError("selection needs at least one candidate")
    fresh = [fresh_count] * n if isinstance(fresh_count, int) else [int(v) for v in fresh_count]
    if len(fresh) != n or min(fresh) < 1:
        raise ValueError("every candidate needs a positive fresh rollout count")
    if not (reward_temperature > 0 and truncation > 0):
        raise ValueError("reward_temperature and truncation have to be positive")
    outer = tuple(candidate_log_ratios) if candidate_log_ratios is not None else (0.0,) * n
    if len(outer) != n or not all(isfinite(v) for v in outer):
        raise ValueError("candidate log-ratios must be finite, one per candidate")
    prefixes = [tuple(prompt) + tuple(generated_prefix) + tuple(c.token_ids) for c in candidates]
    histories = tuple(histories) if histories else tuple(DiffusionReplayHistory(p, ()) for p in prefixes)
    if len(histories) != n or any(h.rollout_prefix != p for h, p in zip(histories, prefixes)):
        raise ValueError("histories must match the candidates one to one")
    replaying = any(h.records for h in histories)
    if replaying:
        if behavior_backend is None or behavior_sampling is None:
            raise ValueError("replayed records need their behaviour backend and policy")
        validate_exact_pair(target_sampling, behavior_sampling)
    tau = reward_temperature
    if rollout_length == 0:
        rewards = _rewards(reward_batch, prompt,
                           [tuple(generated_prefix) + tuple(c.token_ids) for c in candidates], "terminal")
        return _terminal_selection(candidates, outer, rewards, tau, seed)
    seeds = SeedStream(seed)
    cells = _grid(fresh)
    requests = [DiffusionGenerationRequest(prefixes[c], rollout_length, target_sampling,
                                           seeds.derive("dllm-replay-fresh", c, f), f"dllm-replay-fresh:{c}:{f}")
                for c, f in cells]
    drawn = target_backend.sample_batch(requests)
    if len(drawn) != len(requests):
        raise RuntimeError(f"{len(drawn)} fresh rollouts for {len(requests)} requests")
    if any(s.trajectory_logprob is None for s in drawn):
        raise RuntimeError("a fresh rollout came without its trajectory probability")
    own = np.asarray([float(s.trajectory_logprob) for s in drawn])
    behaviour = own
    if replaying:
        behaviour = np.asarray([float(v) for v in behavior_backend.score_trajectories(
            [DiffusionTrajectoryScoreRequest(s, behavior_sampling) for s in drawn])])
        if behaviour.size != len(drawn):
            raise RuntimeError(f"{behaviour.size} behaviour scores for {len(drawn)} fresh rollouts")
    texts = [tuple(generated_prefix) + tuple(candidates[c].token_ids) + tuple(s.token_ids)
             for (c, _), s in zip(cells, drawn)]
    rewards = _rewards(reward_batch, prompt, texts, "fresh")
    rows: list[list[DiffusionReplayRecord]] = [[] for _ in candidates]
    for i, ((c, _), s, r) in enumerate(zip(cells, drawn, rewards)):
        rows[c].append(DiffusionReplayRecord(s.prefix, s, float(own[i]), float(behaviour[i]), r))
    provider = TruncatedReplayRolloutWeightProvider(truncation=truncation, reward_temperature=tau)
    weighted = []
    for cand, history, row, ratio in zip(candidates, histories, rows, outer):
        if history.records:
            estimate = provider.estimate([r.observation for r in history.records], [r.observation for r in row])
        else:
            terms = tuple(r.reward / tau for r in row)
            estimate = ReplayWeightEstimate(logmeanexp(terms), (), terms)
        weighted.append(DiffusionReplayCandidate(cand, estimate, ratio))
    probabilities = normalize_log_weights([c.estimate.log_weight + c.outer_log_ratio for c in weighted])
    pick = int(seeds.generator("dllm-replay-select").choice(n, p=probabilities))
    return DiffusionReplaySelection(tuple(weighted), probabilities, pick, tuple(tuple(row) for row in rows))


__all__ = ["DiffusionReplayCandidate", "DiffusionReplayHistory", "DiffusionReplayRecord",
           "DiffusionReplayRewardBatch", "DiffusionReplaySelection", "build_diffusion_replay_history",
           "select_diffusion_candidates_with_replay", "validate_exact_pair"]
