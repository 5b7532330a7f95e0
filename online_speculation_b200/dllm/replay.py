"""Exact trajectory replay for block-diffusion rollout weights.

Reference behaviour: src/inference_scaling/dllm/replay.py:108-385.  History
rollouts are drawn once from a behaviour policy and scored under the target
policy; a candidate's weight combines truncated-IS history terms
min(c, p/q) exp(r / tau) with fresh target rollouts whose tail correction
(1 - c q/p)+ keeps the estimator unbiased (shared.importance).  Exact
trajectory densities make p/q the ratio of the same reverse trace.
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


def _schedule(s: DiffusionSamplingConfig):
    return s.block_length, s.steps_per_block, s.remasking, s.mask_token_id


def validate_exact_pair(target: DiffusionSamplingConfig, behavior: DiffusionSamplingConfig) -> None:
    if not (target.has_exact_trajectory_density and behavior.has_exact_trajectory_density):
        raise ValueError("replay correction requires exact target and behavior trajectories")
    if _schedule(target) != _schedule(behavior):
        raise ValueError("target and replay behavior trajectory schedules must match")


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


def _rewards(reward_batch, prompt, conts, what: str) -> list[float]:
    vals = [float(v) for v in reward_batch(prompt, conts)]
    if len(vals) != len(conts):
        raise RuntimeError(f"reward evaluator returned an invalid {what} count")
    return vals


def build_diffusion_replay_history(*, target_backend: DiffusionBackend, behavior_backend: DiffusionBackend,
                                   prompt: TokenSequence, generated_prefix: TokenSequence,
                                   candidates: Sequence[DiffusionSample], rollout_length: int,
                                   count_per_candidate: int, target_sampling: DiffusionSamplingConfig,
                                   behavior_sampling: DiffusionSamplingConfig,
                                   reward_batch: DiffusionReplayRewardBatch, seed: int
                                   ) -> tuple[DiffusionReplayHistory, ...]:
    """Draw immutable behaviour trajectories per candidate and precompute their target scores."""
    validate_exact_pair(target_sampling, behavior_sampling)
    if count_per_candidate <= 0:
        raise ValueError("count_per_candidate must be positive")
    prefixes = [prompt + generated_prefix + c.token_ids for c in candidates]
    if rollout_length <= 0:
        return tuple(DiffusionReplayHistory(p, ()) for p in prefixes)
    seeds = SeedStream(seed)
    reqs, owners = [], []
    for ci, p in enumerate(prefixes):
        for hi in range(count_per_candidate):
            reqs.append(DiffusionGenerationRequest(p, rollout_length, behavior_sampling,
                                                   seeds.derive("dllm-replay", ci, hi), f"dllm-replay:{ci}:{hi}"))
            owners.append(ci)
    samples = behavior_backend.sample_batch(reqs)
    if len(samples) != len(reqs):
        raise RuntimeError("behavior backend returned an invalid replay sample count")
    scores = target_backend.score_trajectories([DiffusionTrajectoryScoreRequest(s, target_sampling) for s in samples])
    if len(scores) != len(samples):
        raise RuntimeError("target backend returned an invalid replay score count")
    rewards = _rewards(reward_batch, prompt, [generated_prefix + candidates[o].token_ids + s.token_ids
                                              for o, s in zip(owners, samples)], "replay")
    grouped: list[list[DiffusionReplayRecord]] = [[] for _ in candidates]
    for o, s, t, r in zip(owners, samples, scores, rewards):
        if s.trajectory_logprob is None:
            raise RuntimeError("behavior backend omitted replay trajectory probability")
        grouped[o].append(DiffusionReplayRecord(s.prefix, s, float(t), float(s.trajectory_logprob), r))
    return tuple(DiffusionReplayHistory(p, tuple(g)) for p, g in zip(prefixes, grouped))


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
    """Weight every candidate from fresh rollouts, or corrected replay plus a fresh tail, then draw one."""
    if not candidates:
        raise ValueError("at least one candidate is required")
    n = len(candidates)
    fresh = (fresh_count,) * n if isinstance(fresh_count, int) else tuple(int(v) for v in fresh_count)
    if len(fresh) != n or any(v <= 0 for v in fresh):
        raise ValueError("fresh_count must be positive for every candidate")
    if reward_temperature <= 0 or truncation <= 0:
        raise ValueError("reward_temperature and truncation must be positive")
    outer = tuple(candidate_log_ratios or (0.0,) * n)
    if len(outer) != n or not all(isfinite(v) for v in outer):
        raise ValueError("candidate log-ratios must be finite and match the candidates")
    prefixes = [prompt + generated_prefix + c.token_ids for c in candidates]
    histories = histories or tuple(DiffusionReplayHistory(p, ()) for p in prefixes)
    if len(histories) != n:
        raise ValueError("one replay history is required per candidate")
    replay = any(h.records for h in histories)
    if replay:
        if behavior_backend is None or behavior_sampling is None:
            raise ValueError("replay records require their behavior backend and policy")
        validate_exact_pair(target_sampling, behavior_sampling)
    tau = reward_temperature
    if rollout_length == 0:
        rewards = _rewards(reward_batch, prompt, [generated_prefix + c.token_ids for c in candidates], "terminal")
        cands = tuple(DiffusionReplayCandidate(c, ReplayWeightEstimate(r / tau, (), (r / tau,)), o)
                      for c, r, o in zip(candidates, rewards, outer))
        probs = normalize_log_weights([c.estimate.log_weight + c.outer_log_ratio for c in cands])
        return DiffusionReplaySelection(cands, probs, int(np.random.default_rng(seed).choice(n, p=probs)),
                                        tuple(() for _ in candidates))
    seeds = SeedStream(seed)
    reqs, owners = [], []
    for ci, p in enumerate(prefixes):
        if histories[ci].rollout_prefix != p:
            raise ValueError("replay history does not belong to its candidate")
        for fi in range(fresh[ci]):
            reqs.append(DiffusionGenerationRequest(p, rollout_length, target_sampling,
                                                   seeds.derive("dllm-replay-fresh", ci, fi),
                                                   f"dllm-replay-fresh:{ci}:{fi}"))
            owners.append(ci)
    samples = target_backend.sample_batch(reqs)
    if len(samples) != len(reqs):
        raise RuntimeError("target backend returned an invalid fresh rollout count")
    if replay:
        beh = [float(v) for v in behavior_backend.score_trajectories(
            [DiffusionTrajectoryScoreRequest(s, behavior_sampling) for s in samples])]
        if len(beh) != len(samples):
            raise RuntimeError("behavior backend returned an invalid fresh score count")
    else:
        beh = [None] * len(samples)
    rewards = _rewards(reward_batch, prompt, [generated_prefix + candidates[o].token_ids + s.token_ids
                                              for o, s in zip(owners, samples)], "fresh rollout")
    grouped: list[list[DiffusionReplayRecord]] = [[] for _ in candidates]
    for o, s, b, r in zip(owners, samples, beh, rewards):
        if s.trajectory_logprob is None:
            raise RuntimeError("target backend omitted fresh trajectory probability")
        grouped[o].append(DiffusionReplayRecord(s.prefix, s, float(s.trajectory_logprob),
                                                float(b) if b is not None else float(s.trajectory_logprob), r))
    provider = TruncatedReplayRolloutWeightProvider(truncation=truncation, reward_temperature=tau)
    cands = []
    for c, h, f, o in zip(candidates, histories, grouped, outer):
        if h.records:
            est = provider.estimate([r.observation for r in h.records], [r.observation for r in f])
        else:
            terms = tuple(r.reward / tau for r in f)
            est = ReplayWeightEstimate(logmeanexp(terms), (), terms)
        cands.append(DiffusionReplayCandidate(c, est, o))
    probs = normalize_log_weights([c.estimate.log_weight + c.outer_log_ratio for c in cands])
    sel = int(seeds.generator("dllm-replay-select").choice(n, p=probs))
    return DiffusionReplaySelection(tuple(cands), probs, sel, tuple(tuple(g) for g in grouped))


__all__ = ["DiffusionReplayCandidate", "DiffusionReplayHistory", "DiffusionReplayRecord",
           "DiffusionReplayRewardBatch", "DiffusionReplaySelection", "build_diffusion_replay_history",
           "select_diffusion_candidates_with_replay", "validate_exact_pair"]
