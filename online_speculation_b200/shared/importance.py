"""Importance weights for rollouts and truncated-history replay.

* on/off-policy conditional weights: log w = r / tau (+ log p - log q, optionally
  clipped), combined over rollouts with log-mean-exp;
* truncated replay: history terms min(log c, log p/b) + r/tau plus an exact
  fresh-sample tail correction log(1 - c b/p) that keeps the estimator unbiased.
Reference: src/inference_scaling/shared/importance.py:51-228.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import exp, isfinite, log, log1p
from typing import Generic, Literal, TypeVar

import numpy as np

from .metrics import importance_effective_sample_size

PayloadT = TypeVar("PayloadT")


def logmeanexp(values: Sequence[float]) -> float:
    if not len(values):
        raise ValueError("at least one value is required")
    top = max(values)
    if top == float("-inf"):
        return top
    return top + log(sum(exp(v - top) for v in values)) - log(len(values))


@dataclass(frozen=True, slots=True)
class RolloutObservation(Generic[PayloadT]):
    reward: float
    target_logprob: float | None = None
    proposal_logprob: float | None = None
    payload: PayloadT | None = None

    def __post_init__(self) -> None:
        if not isfinite(self.reward):
            raise ValueError("rollout reward must be finite")
        for name in ("target_logprob", "proposal_logprob"):
            value = getattr(self, name)
            if value is not None and not isfinite(value):
                raise ValueError(f"{name} must be finite when provided")


@dataclass(frozen=True, slots=True)
class WeightedRollout(Generic[PayloadT]):
    observation: RolloutObservation[PayloadT]
    raw_log_importance_ratio: float | None
    applied_log_importance_ratio: float | None
    log_weight: float


@dataclass(frozen=True, slots=True)
class MonteCarloWeightEstimate(Generic[PayloadT]):
    log_weight: float
    rollouts: tuple[WeightedRollout[PayloadT], ...]


class MonteCarloRolloutWeightProvider(Generic[PayloadT]):
    def __init__(self, *, reward_temperature: float,
                 correction: Literal["importance", "identity", "none"] = "importance",
                 log_ratio_clip: float | None = None) -> None:
        if reward_temperature <= 0:
            raise ValueError("reward_temperature must be positive")
        if correction not in ("importance", "identity", "none"):
            raise ValueError(f"unknown rollout correction mode {correction!r}")
        if log_ratio_clip is not None and log_ratio_clip <= 0:
            raise ValueError("log_ratio_clip must be positive when provided")
        if correction != "importance" and log_ratio_clip is not None:
            raise ValueError("log-ratio clipping requires importance correction")
        self.reward_temperature = float(reward_temperature)
        self.correction = correction
        self.log_ratio_clip = log_ratio_clip

    def weight(self, obs: RolloutObservation[PayloadT]) -> WeightedRollout[PayloadT]:
        raw = applied = None
        if self.correction == "importance":
            if obs.target_logprob is None or obs.proposal_logprob is None:
                raise ValueError("importance correction requires target and proposal log-probabilities")
            raw = applied = obs.target_logprob - obs.proposal_logprob
            if self.log_ratio_clip is not None:
                applied = min(max(raw, -self.log_ratio_clip), self.log_ratio_clip)
        elif self.correction == "identity":
            raw = applied = 0.0
        log_w = obs.reward / self.reward_temperature + (applied or 0.0)
        return WeightedRollout(obs, raw, applied, log_w)

    def estimate(self, observations: Sequence[RolloutObservation[PayloadT]]) -> MonteCarloWeightEstimate[PayloadT]:
        weighted = tuple(self.weight(o) for o in observations)
        if not weighted:
            raise ValueError("at least one rollout is required to estimate a conditional weight")
        return MonteCarloWeightEstimate(logmeanexp([w.log_weight for w in weighted]), weighted)


@dataclass(frozen=True, slots=True)
class ProbabilityObservation:
    target_logprob: float
    behavior_logprob: float
    reward: float


def corrected_replay_log_weight(history: Sequence[ProbabilityObservation], fresh: Sequence[ProbabilityObservation], *,
                                truncation: float, reward_temperature: float
                                ) -> tuple[float, tuple[float, ...], tuple[float, ...]]:
    if not history:
        raise ValueError("corrected replay requires at least one history observation")
    if not fresh:
        raise ValueError("corrected replay requires at least one fresh observation")
    if truncation <= 0 or reward_temperature <= 0:
        raise ValueError("truncation and reward_temperature must be positive")
    log_c = log(truncation)
    hist: list[float] = []
    for o in history:
        ratio = o.target_logprob - o.behavior_logprob
        if not isfinite(ratio):
            raise ValueError("history behavior support must lie inside target support")
        hist.append(min(log_c, ratio) + o.reward / reward_temperature)
    tail: list[float] = []
    for o in fresh:
        if o.behavior_logprob == float("-inf"):
            term = 0.0
        else:
            ratio = o.target_logprob - o.behavior_logprob
            term = float("-inf") if ratio <= log_c else log1p(-exp(log_c - ratio))
        tail.append(term + o.reward / reward_temperature)
    finite = [t for t in tail if t != float("-inf")]
    fresh_mean = logmeanexp(finite) + log(len(finite) / len(tail)) if finite else float("-inf")
    return float(np.logaddexp(logmeanexp(hist), fresh_mean)), tuple(hist), tuple(tail)


@dataclass(frozen=True, slots=True)
class ReplayWeightEstimate:
    log_weight: float
    history_log_terms: tuple[float, ...]
    fresh_log_terms: tuple[float, ...]

    @property
    def history_count(self) -> int:
        return len(self.history_log_terms)

    @property
    def fresh_count(self) -> int:
        return len(self.fresh_log_terms)

    @property
    def history_ess(self) -> float:
        return importance_effective_sample_size(self.history_log_terms)

    @property
    def fresh_ess(self) -> float:
        return importance_effective_sample_size(tuple(v for v in self.fresh_log_terms if isfinite(v)))


class TruncatedReplayRolloutWeightProvider:
    def __init__(self, *, truncation: float, reward_temperature: float) -> None:
        if truncation <= 0 or reward_temperature <= 0:
            raise ValueError("truncation and reward_temperature must be positive")
        self.truncation = float(truncation)
        self.reward_temperature = float(reward_temperature)

    def estimate(self, history, fresh) -> ReplayWeightEstimate:
        return ReplayWeightEstimate(*corrected_replay_log_weight(
            history, fresh, truncation=self.truncation, reward_temperature=self.reward_temperature))
