"""Streaming importance sampling with a fresh design frozen in advance.

History contributions may be revealed, and looked at, before the fresh budget is
fixed.  ``freeze`` then names, per candidate, the fresh sample ids that will enter
the estimate; afterwards exactly those ids are accepted, each once, in any order.
The estimate of a candidate is the log-mean-exp of its contributions, so arrival
order changes what an update callback sees along the way, never the final
statistic.  Contributions live in one flat ledger (id -> candidate, source, weight)
whose per-candidate summaries are recomputed on demand.  The selection stream is
``("frozen-streaming-is", *labels)``, as in
src/inference_scaling/experimental/arllm/streaming_is.py.
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
    if not reward_temperature > 0:
        raise ValueError("reward_temperature has to be positive")
    terms = np.asarray([reward, target_logprob, behavior_logprob], dtype=np.float64)
    if not np.isfinite(terms).all():
        raise ValueError("reward and log-probabilities have to be finite")
    return float(terms[0] / reward_temperature + terms[1] - terms[2])


@dataclass(frozen=True, slots=True)
class ISContribution:
    sample_id: str
    candidate_index: int
    log_weight: float
    source: str

    def __post_init__(self) -> None:
        if not self.sample_id or self.candidate_index < 0 or not isfinite(self.log_weight) or \
                self.source not in ("history", "fresh"):
            raise ValueError(f"invalid contribution {self.sample_id!r}: needs an id, a candidate index >= 0, "
                             "a finite log weight and source 'history' or 'fresh'")


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
        if candidate_count < 1:
            raise ValueError("the estimator needs at least one candidate")
        self.candidate_count = int(candidate_count)
        self._lock = threading.RLock()
        self._on_update = on_update
        self._ledger: dict[str, ISContribution] = {}       # arrival order is kept
        self._design: dict[str, int] | None = None

    @property
    def frozen(self) -> bool:
        with self._lock:
            return self._design is not None

    def _fresh_received(self) -> int:
        return sum(c.source == "fresh" for c in self._ledger.values())

    @property
    def complete(self) -> bool:
        with self._lock:
            return self._design is not None and self._fresh_received() == len(self._design)

    def _check_candidate(self, index: int) -> None:
        if not 0 <= index < self.candidate_count:
            raise ValueError(f"candidate {index} is outside 0..{self.candidate_count - 1}")

    def _record(self, contribution: ISContribution) -> None:
        self._check_candidate(contribution.candidate_index)
        if contribution.sample_id in self._ledger:
            raise ValueError(f"sample {contribution.sample_id!r} already contributed")
        self._ledger[contribution.sample_id] = contribution
        if self._on_update is None:
            return
        try:
            self._on_update(self.snapshot(), contribution)
        except BaseException:
            del self._ledger[contribution.sample_id]      # a failing observer leaves no trace
            raise

    def add_history(self, sample_id: str, candidate_index: int, log_weight: float) -> None:
        with self._lock:
            if self._design is not None:
                raise RuntimeError("history has to be revealed before the fresh design is frozen")
            self._record(ISContribution(sample_id, int(candidate_index), float(log_weight), "history"))

    def freeze(self, fresh_sample_ids: Sequence[Sequence[str]]) -> FrozenISSnapshot:
        with self._lock:
            if self._design is not None:
                raise RuntimeError("the fresh design was already frozen")
            if len(fresh_sample_ids) != self.candidate_count:
                raise ValueError(f"{len(fresh_sample_ids)} id lists for {self.candidate_count} candidates")
            has_history = {c.candidate_index for c in self._ledger.values()}
            design: dict[str, int] = {}
            for k, ids in enumerate(fresh_sample_ids):
                if not ids and k not in has_history:
                    raise ValueError(f"candidate {k} would have neither history nor fresh samples")
                for sid in ids:
                    if not sid or sid in design or sid in self._ledger:
                        raise ValueError(f"fresh sample id {sid!r} is empty or not unique")
                    design[sid] = k
            self._design = design
            return self.snapshot()

    def consume_fresh(self, sample_id: str, candidate_index: int, log_weight: float) -> None:
        with self._lock:
            if self._design is None:
                raise RuntimeError("fresh samples are accepted only after the design is frozen")
            if sample_id not in self._design:
                raise ValueError(f"{sample_id!r} is not part of the frozen fresh design")
            if self._design[sample_id] != candidate_index:
                raise ValueError(f"{sample_id!r} belongs to candidate {self._design[sample_id]}, "
                                 f"not {candidate_index}")
            self._record(ISContribution(sample_id, int(candidate_index), float(log_weight), "fresh"))

    def _weights_of(self, candidate: int) -> list[float]:
        return [c.log_weight for c in self._ledger.values() if c.candidate_index == candidate]

    def snapshot(self) -> FrozenISSnapshot:
        with self._lock:
            per = [self._weights_of(k) for k in range(self.candidate_count)]
            return FrozenISSnapshot(
                frozen=self._design is not None, complete=self.complete,
                expected_fresh=len(self._design or {}), received_fresh=self._fresh_received(),
                history_count=sum(c.source == "history" for c in self._ledger.values()),
                log_weights=tuple(logmeanexp(w) if w else float("-inf") for w in per),
                effective_sample_sizes=tuple(importance_effective_sample_size(w) for w in per),
                contribution_counts=tuple(len(w) for w in per))

    def final_log_weights(self) -> tuple[float, ...]:
        with self._lock:
            if not self.complete:
                raise RuntimeError("not every frozen fresh sample has arrived yet")
            return self.snapshot().log_weights

    def select(self, seeds: SeedStream, *labels: object) -> int:
        weights = np.asarray(self.final_log_weights(), dtype=np.float64)
        if not np.isfinite(weights).all():
            raise RuntimeError("some candidate has no finite estimate")
        p = np.exp(weights - weights.max())
        return int(seeds.generator("frozen-streaming-is", *labels).choice(self.candidate_count, p=p / p.sum()))

    def contributions(self, candidate_index: int) -> tuple[ISContribution, ...]:
        with self._lock:
            self._check_candidate(candidate_index)
            return tuple(c for c in self._ledger.values() if c.candidate_index == candidate_index)


__all__ = ["FrozenISSnapshot", "FrozenStreamingISEstimator", "ISContribution", "ISUpdateCallback",
           "ordinary_importance_log_weight"]
