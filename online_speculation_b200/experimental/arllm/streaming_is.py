"""Streaming importance sampling with a frozen fresh design.

History contributions may be revealed (and inspected) before the fresh budget
is fixed.  ``freeze`` declares, per candidate, the ids of the fresh samples
that will enter the estimate; afterwards only those ids are accepted, each
exactly once, in any arrival order.  The final per-candidate estimate is the
log-mean-exp of its contributions, so arrival order changes wall-clock
behaviour (when a callback sees which snapshot) but never the statistic.

Reference behaviour: src/inference_scaling/experimental/arllm/streaming_is.py:22-226.
"""

from __future__ import annotations

import threading
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from math import isfinite

import numpy as np

from ...shared.importance import logmeanexp
from ...shared.metrics import importance_effective_sample_size
from ...shared.rng import SeedStream


def ordinary_importance_log_weight(*, reward: float, reward_temperature: float, target_logprob: float,
                                   behavior_logprob: float) -> float:
    """Unclipped log contribution r / tau + log p_target - log p_behaviour."""
    if reward_temperature <= 0:
        raise ValueError("reward_temperature must be positive")
    if not all(isfinite(float(v)) for v in (reward, target_logprob, behavior_logprob)):
        raise ValueError("importance-sampling inputs must be finite")
    return float(reward) / reward_temperature + float(target_logprob) - float(behavior_logprob)


@dataclass(frozen=True, slots=True)
class ISContribution:
    sample_id: str
    candidate_index: int
    log_weight: float
    source: str

    def __post_init__(self) -> None:
        if not self.sample_id:
            raise ValueError("IS sample id cannot be empty")
        if self.candidate_index < 0:
            raise ValueError("candidate index must be non-negative")
        if not isfinite(self.log_weight):
            raise ValueError("IS log weight must be finite")
        if self.source not in ("history", "fresh"):
            raise ValueError("IS contribution source must be history or fresh")


@dataclass(frozen=True, slots=True)
class FrozenISSnapshot:
    frozen: bool
    complete: bool
    expected_fresh: int
    received_fresh: int
    history_count: int
    log_weights: tuple[float, ...]
    effective_sample_sizes: tuple[float, ...]
    contribution_counts: tuple[int, ...]


ISUpdateCallback = Callable[[FrozenISSnapshot, ISContribution], None]


class FrozenStreamingISEstimator:
    def __init__(self, candidate_count: int, *, on_update: ISUpdateCallback | None = None):
        if candidate_count <= 0:
            raise ValueError("candidate_count must be positive")
        self.candidate_count = int(candidate_count)
        self._lock = threading.RLock()
        self._on_update = on_update
        self._groups: list[list[ISContribution]] = [[] for _ in range(self.candidate_count)]
        self._ids: set[str] = set()
        self._design: dict[str, int] | None = None
        self._fresh_seen: set[str] = set()

    @property
    def frozen(self) -> bool:
        with self._lock:
            return self._design is not None

    @property
    def complete(self) -> bool:
        with self._lock:
            return self._design is not None and len(self._fresh_seen) == len(self._design)

    def _add(self, c: ISContribution) -> None:
        if not 0 <= c.candidate_index < self.candidate_count:
            raise ValueError("candidate index is outside the estimator")
        if c.sample_id in self._ids:
            raise ValueError(f"duplicate IS sample id {c.sample_id!r}")
        group = self._groups[c.candidate_index]
        self._ids.add(c.sample_id)
        group.append(c)
        if self._on_update is not None:
            try:
                self._on_update(self.snapshot(), c)
            except BaseException:
                # a failing observer leaves the estimator as it was
                group.pop()
                self._ids.discard(c.sample_id)
                raise

    def add_history(self, sample_id: str, candidate_index: int, log_weight: float) -> None:
        with self._lock:
            if self._design is not None:
                raise RuntimeError("history cannot be revealed after the fresh design is frozen")
            self._add(ISContribution(sample_id, int(candidate_index), float(log_weight), "history"))

    def freeze(self, fresh_sample_ids: Sequence[Sequence[str]]) -> FrozenISSnapshot:
        with self._lock:
            if self._design is not None:
                raise RuntimeError("fresh IS design is already frozen")
            if len(fresh_sample_ids) != self.candidate_count:
                raise ValueError("fresh design needs one id list per candidate")
            design: dict[str, int] = {}
            for k, ids in enumerate(fresh_sample_ids):
                if not ids and not self._groups[k]:
                    raise ValueError("every candidate needs history or a fresh evaluation")
                for sid in ids:
                    if not sid:
                        raise ValueError("fresh IS sample id cannot be empty")
                    if sid in design or sid in self._ids:
                        raise ValueError(f"duplicate frozen IS sample id {sid!r}")
                    design[sid] = k
            self._design = design
            return self.snapshot()

    def consume_fresh(self, sample_id: str, candidate_index: int, log_weight: float) -> None:
        with self._lock:
            if self._design is None:
                raise RuntimeError("fresh contribution arrived before the design was frozen")
            owner = self._design.get(sample_id)
            if owner is None:
                raise ValueError(f"fresh sample id {sample_id!r} is not in the frozen design")
            if owner != candidate_index:
                raise ValueError("fresh contribution belongs to a different candidate")
            if sample_id in self._fresh_seen:
                raise ValueError(f"duplicate IS sample id {sample_id!r}")
            self._fresh_seen.add(sample_id)
            try:
                self._add(ISContribution(sample_id, int(candidate_index), float(log_weight), "fresh"))
            except BaseException:
                self._fresh_seen.discard(sample_id)
                raise

    def snapshot(self) -> FrozenISSnapshot:
        with self._lock:
            lw = tuple(logmeanexp([c.log_weight for c in g]) if g else float("-inf") for g in self._groups)
            return FrozenISSnapshot(
                self._design is not None, self.complete, len(self._design or {}), len(self._fresh_seen),
                sum(c.source == "history" for g in self._groups for c in g), lw,
                tuple(importance_effective_sample_size([c.log_weight for c in g]) for g in self._groups),
                tuple(len(g) for g in self._groups))

    def final_log_weights(self) -> tuple[float, ...]:
        with self._lock:
            if not self.complete:
                raise RuntimeError("fresh IS design is not complete")
            return self.snapshot().log_weights

    def select(self, seeds: SeedStream, *labels: object) -> int:
        lw = np.asarray(self.final_log_weights(), dtype=np.float64)
        if not np.all(np.isfinite(lw)):
            raise RuntimeError("every candidate needs a finite final IS estimate")
        p = np.exp(lw - lw.max())
        return int(seeds.generator("frozen-streaming-is", *labels).choice(self.candidate_count, p=p / p.sum()))

    def contributions(self, candidate_index: int) -> tuple[ISContribution, ...]:
        with self._lock:
            if not 0 <= candidate_index < self.candidate_count:
                raise ValueError("candidate index is outside the estimator")
            return tuple(self._groups[candidate_index])


__all__ = ["FrozenISSnapshot", "FrozenStreamingISEstimator", "ISContribution", "ISUpdateCallback",
           "ordinary_importance_log_weight"]
