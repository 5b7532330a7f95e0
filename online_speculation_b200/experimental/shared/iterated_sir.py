"""Iterated sampling-importance-resampling (i-SIR).

One transition puts the current weighted state in slot 0 of a pool, fills the other
slots with fresh states drawn independently from the same extended proposal, and
keeps one slot chosen in proportion to the weights.  Because the current state is
kept with everything its weight was computed from, the kernel leaves the target
invariant for any pool size.

Mixing: with L = sup w / E_q[w] and pool size N the kernel is minorised with
constant eps = (N - 1) / (2 L + N - 2), so after k transitions the total variation
to the target is at most (1 - eps)^k.  Public names follow
src/inference_scaling/experimental/shared/iterated_sir.py.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
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
        n = len(self.pool)
        if n < 2:
            raise ValueError("an i-SIR pool holds the current state and at least one fresh state")
        if self.pool[0] is not self.previous:
            raise ValueError("slot 0 of the pool is the current state")
        if len(self.probabilities) != n or not 0 <= self.selected_index < n:
            raise ValueError("probabilities and the selected index must match the pool")

    @property
    def selected(self) -> StepwiseCandidate[StateT]:
        return self.pool[self.selected_index]

    @property
    def retained_previous(self) -> bool:
        return self.selected_index == 0


def iterated_sir_transition(current: StepwiseCandidate[StateT], fresh: Sequence[StepwiseCandidate[StateT]], *,
                            rng: np.random.Generator) -> IteratedSIRTransition[StateT]:
    pool = (current, *fresh)
    if len(pool) < 2:
        raise ValueError("an i-SIR transition needs at least one fresh state")
    probabilities = normalize_log_weights([state.log_weight for state in pool])
    choice = int(rng.choice(len(pool), p=probabilities))
    return IteratedSIRTransition(current, pool, probabilities, choice)


def iterated_sir_tv_bound(*, pool_size: int, updates: int, normalized_weight_supremum: float) -> float:
    if isinstance(pool_size, bool) or not isinstance(pool_size, (int, np.integer)) or pool_size < 2:
        raise ValueError("pool_size is an integer of at least 2")
    if isinstance(updates, bool) or not isinstance(updates, (int, np.integer)) or updates < 0:
        raise ValueError("updates is a non-negative integer")
    sup = float(normalized_weight_supremum)
    if not np.isfinite(sup) or sup < 1.0:
        raise ValueError("the normalised weight supremum is finite and at least 1")
    eps = (pool_size - 1) / (2.0 * sup + pool_size - 2)
    return float(np.power(1.0 - eps, updates))


__all__ = ["IteratedSIRTransition", "iterated_sir_transition", "iterated_sir_tv_bound"]
