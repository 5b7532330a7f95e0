"""Importance weights of rollouts and of truncated-history replay.

Everything is computed on float64 arrays:

* conditional rollout weights ``log w_i = r_i / tau + c_i`` where the correction
  ``c_i`` is the (optionally clipped) log ratio ``log p_i - log q_i`` ("importance"),
  zero ("identity", reported as a ratio of 0) or absent ("none"); a set of rollouts
  is summarised by the log of the mean weight;
* truncated replay of old rollouts drawn from a behaviour policy b: every history
  term is ``min(log c, log p/b) + r / tau`` and every fresh draw contributes the
  exact tail correction ``log(1 - c b/p) + r / tau`` (zero mass where p <= c b), so
  history and fresh parts together are unbiased for the target.

The public names and fields follow src/inference_scaling/shared/importance.py,
whose estimators the algorithms are specified against.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Generic, Literal, TypeVar

import numpy as np

from .metrics import importance_effective_sample_size

PayloadT = TypeVar("PayloadT")

_NEG_INF = float("-inf")


def _logmeanexp_array(v: np.ndarray) -> float:
    if v.size == 0:
        raise ValueError("log-mean-exp of an empty set is undefined")
    top = float(v.max())
    if top == _NEG_INF:
        return _NEG_INF
    return top + float(np.log(np.exp(v - top).mean()))


def logmeanexp(values: Sequence[float]) -> float:
    """log(mean(exp(values))) without overflow; -inf when every value is -inf."""
    return _logmeanexp_array(np.asarray(list(values), dtype=np.float64))


def _finite_or_none(name: str, value: float | None) -> None:
    if value is not None and not np.isfinite(value):
        raise ValueError(f"{name} has to be a finite number when it is given")


@dataclass(frozen=True, slots=True)
class RolloutObservation(Generic[PayloadT]):
    reward: float
    target_logprob: float | None = None
    proposal_logprob: float | None = None
    payload: PayloadT | None = None

    def __post_init__(self) -> None:
        if not np.isfinite(self.reward):
            raise ValueError("a rollout reward has to be finite")
        _finite_or_none("target_logprob", self.target_logprob)
        _finite_or_none("proposal_logprob", self.proposal_logprob)


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
    """log w = r / tau + correction, averaged over the rollouts of one candidate."""

    _MODES = ("importance", "identity", "none")

    def __init__(self, *, reward_temperature: float,
                 correction: Literal["importance", "identity", "none"] = "importance",
                 log_ratio_clip: float | None = None) -> None:
        if not reward_temperature > 0:
            raise ValueError("reward_temperature has to be positive")
        if correction not in self._MODES:
            raise ValueError(f"correction must be one of {self._MODES}, got {correction!r}")
        if log_ratio_clip is not None and not log_ratio_clip > 0:
            raise ValueError("log_ratio_clip has to be positive")
        if log_ratio_clip is not None and correction != "importance":
            raise ValueError("clipping applies to importance ratios only (correction='importance')")
        self.reward_temperature = float(reward_temperature)
        self.correction = correction
        self.log_ratio_clip = log_ratio_clip

    def _ratios(self, observations: Sequence[RolloutObservation]) -> tuple[np.ndarray | None, np.ndarray | None]:
        n = len(observations)
        if self.correction == "none":
            return None, None
        if self.correction == "identity":
            z = np.zeros(n)
            return z, z
        p = [o.target_logprob for o in observations]
        q = [o.proposal_logprob for o in observations]
        if any(v is None for v in p) or any(v is None for v in q):
            raise ValueError("importance correction needs both target and proposal log-probabilities")
        raw = np.asarray(p, dtype=np.float64) - np.asarray(q, dtype=np.float64)
        if self.log_ratio_clip is None:
            return raw, raw
        return raw, np.clip(raw, -self.log_ratio_clip, self.log_ratio_clip)

    def _weigh_all(self, observations: Sequence[RolloutObservation[PayloadT]]) -> tuple[WeightedRollout, ...]:
        raw, applied = self._ratios(observations)
        rewards = np.fromiter((o.reward for o in observations), dtype=np.float64, count=len(observations))
        log_w = rewards / self.reward_temperature + (0.0 if applied is None else applied)
        out = []
        for i, o in enumerate(observations):
            out.append(WeightedRollout(o, None if raw is None else float(raw[i]),
                                       None if applied is None else float(applied[i]), float(log_w[i])))
        return tuple(out)

    def weight(self, obs: RolloutObservation[PayloadT]) -> WeightedRollout[PayloadT]:
        return self._weigh_all([obs])[0]

    def estimate(self, observations: Sequence[RolloutObservation[PayloadT]]) -> MonteCarloWeightEstimate[PayloadT]:
        if not len(observations):
            raise ValueError("a conditional weight needs at least one rollout")
        weighted = self._weigh_all(list(observations))
        log_w = np.fromiter((w.log_weight for w in weighted), dtype=np.float64, count=len(weighted))
        return MonteCarloWeightEstimate(_logmeanexp_array(log_w), weighted)


@dataclass(frozen=True, slots=True)
class ProbabilityObservation:
    target_logprob: float
    behavior_logprob: float
    reward: float


def _columns(observations: Sequence[ProbabilityObservation]) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    arr = np.asarray([(o.target_logprob, o.behavior_logprob, o.reward) for o in observations], dtype=np.float64)
    return arr[:, 0], arr[:, 1], arr[:, 2]


def corrected_replay_log_weight(history: Sequence[ProbabilityObservation], fresh: Sequence[ProbabilityObservation], *,
                                truncation: float, reward_temperature: float
                                ) -> tuple[float, tuple[float, ...], tuple[float, ...]]:
    """(log weight, per-history terms, per-fresh terms) of the truncated replay estimator."""
    if not len(history) or not len(fresh):
        raise ValueError("truncated replay needs at least one history and one fresh observation")
    if not (truncation > 0 and reward_temperature > 0):
        raise ValueError("truncation and reward_temperature have to be positive")
    log_c = float(np.log(truncation))
    p_h, b_h, r_h = _columns(history)
    ratio_h = p_h - b_h
    if not np.isfinite(ratio_h).all():
        raise ValueError("a history draw lies outside the target's support (non-finite log p - log b)")
    hist = np.minimum(log_c, ratio_h) + r_h / reward_temperature
    p_f, b_f, r_f = _columns(fresh)
    with np.errstate(invalid="ignore", divide="ignore"):
        ratio_f = p_f - b_f
        # behaviour mass zero: no history can stand for this draw, the full draw counts
        tail = np.where(b_f == _NEG_INF, 0.0,
                        np.where(ratio_f <= log_c, _NEG_INF, np.log1p(-np.exp(log_c - ratio_f))))
    tail = tail + r_f / reward_temperature
    finite = np.isfinite(tail)
    if finite.any():
        fresh_part = _logmeanexp_array(tail[finite]) + float(np.log(finite.mean()))
    else:
        fresh_part = _NEG_INF
    total = float(np.logaddexp(_logmeanexp_array(hist), fresh_part))
    return total, tuple(float(v) for v in hist), tuple(float(v) for v in tail)


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
        terms = np.asarray(self.fresh_log_terms, dtype=np.float64)
        return importance_effective_sample_size(tuple(terms[np.isfinite(terms)]))


class TruncatedReplayRolloutWeightProvider:
    """Estimator object over :func:`corrected_replay_log_weight` with fixed c and tau."""

    def __init__(self, *, truncation: float, reward_temperature: float) -> None:
        if not (truncation > 0 and reward_temperature > 0):
            raise ValueError("truncation and reward_temperature have to be positive")
        self.truncation = float(truncation)
        self.reward_temperature = float(reward_temperature)

    def estimate(self, history, fresh) -> ReplayWeightEstimate:
        total, hist, tail = corrected_replay_log_weight(history, fresh, truncation=self.truncation,
                                                        reward_temperature=self.reward_temperature)
        return ReplayWeightEstimate(total, hist, tail)
