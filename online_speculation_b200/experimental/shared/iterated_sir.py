"""Iterated sampling-importance-resampling (i-SIR) transition.

One transition keeps the current weighted state in pool slot 0, adds fresh
states drawn independently from the same extended proposal, and resamples one
slot in proportion to the weights.  Retaining the full current state (with all
auxiliary variables behind its weight) makes the kernel invariant for the
target, for any pool size.

``iterated_sir_tv_bound``: with L = sup w / E_q[w] and pool size N the kernel
satisfies a minorisation with constant eps = (N - 1) / (2 L + N - 2), so the
total variation after k updates is at most (1 - eps)^k.

Reference behaviour: src/inference_scaling/experimental/shared/iterated_sir.py:17-103.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import isfinite
from typing import Generic, TypeVar

import numpy as np

from ...shared.stepwise import StepwiseCandidate, normalize_log_weights

StateT = TypeVar("StateT")


@dataclass(frozen=True, slots=True)
class IteratedSIRTransition(Generic[StateT]):
    previous: StepwiseCandidate[StateT]
    pool: tuple[StepwiseCandidate[StateT], ...]
    probabilities: tuple[float, ...]
    selected_index: int

    def __post_init__(self) -> None:
        if len(self.pool) < 2:
            raise ValueError("an i-SIR pool requires at least two states")
        if self.pool[0] is not self.previous:
            raise ValueError("pool slot zero must hold the previous state")
        if len(self.probabilities) != len(self.pool):
            raise ValueError("each pool state needs one probability")
        if not 0 <= self.selected_index < len(self.pool):
            raise ValueError("selected_index lies outside the pool")

    @property
    def selected(self) -> StepwiseCandidate[StateT]:
        return self.pool[self.selected_index]

    @property
    def retained_previous(self) -> bool:
        return self.selected_index == 0


def iterated_sir_transition(current: StepwiseCandidate[StateT], fresh: Sequence[StepwiseCandidate[StateT]], *,
                            rng: np.random.Generator) -> IteratedSIRTransition[StateT]:
    fresh = tuple(fresh)
    if not fresh:
        raise ValueError("an i-SIR transition requires at least one fresh state")
    pool = (current,) + fresh
    probs = normalize_log_weights([c.log_weight for c in pool])
    return IteratedSIRTransition(current, pool, probs, int(rng.choice(len(pool), p=probs)))


def iterated_sir_tv_bound(*, pool_size: int, updates: int, normalized_weight_supremum: float) -> float:
    if isinstance(pool_size, bool) or pool_size < 2:
        raise ValueError("pool_size must be an integer of at least two")
    if isinstance(updates, bool) or updates < 0:
        raise ValueError("updates must be a non-negative integer")
    L = float(normalized_weight_supremum)
    if not isfinite(L) or L < 1:
        raise ValueError("normalized_weight_supremum must be finite and at least one")
    eps = (pool_size - 1) / (2.0 * L + pool_size - 2)
    return float((1.0 - eps) ** updates)


__all__ = ["IteratedSIRTransition", "iterated_sir_transition", "iterated_sir_tv_bound"]
