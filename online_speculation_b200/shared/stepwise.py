"""Sequential importance resampling over opaque generation states.

A :class:`StepwiseSampler` owns a backend (propose / evaluate / advance /
is_terminal) and a seed stream.  Each step asks the backend for proposals,
has it score them into weighted candidates, keeps one candidate drawn in
proportion to its weight, and advances the state with it.  The draw uses one
explicit uniform from the stream ``(*namespace, step, "select")``, so a run is a
pure function of the root seed.  The module-level functions keep the call
signatures of src/inference_scaling/shared/stepwise.py, which the conditional-IS
algorithms are written against.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Generic, Protocol, TypeVar, runtime_checkable

import numpy as np

from .rng import SeedStream
from .smc import normalize_smc_log_weights

StateT = TypeVar("StateT")
ProposalT = TypeVar("ProposalT")
CandidateT = TypeVar("CandidateT")


@dataclass(frozen=True, slots=True)
class StepwiseCandidate(Generic[CandidateT]):
    value: CandidateT
    log_weight: float
    diagnostics: dict | None = None


@dataclass(frozen=True, slots=True)
class StepwiseSelection(Generic[StateT, CandidateT]):
    step_index: int
    state_before: StateT
    candidates: tuple[StepwiseCandidate[CandidateT], ...]
    probabilities: tuple[float, ...]
    selected_index: int

    @property
    def selected(self) -> StepwiseCandidate[CandidateT]:
        return self.candidates[self.selected_index]


@dataclass(frozen=True, slots=True)
class StepwiseGenerationResult(Generic[StateT, CandidateT]):
    final_state: StateT
    steps: tuple[StepwiseSelection[StateT, CandidateT], ...]


@runtime_checkable
class StepwiseGenerationBackend(Protocol[StateT, ProposalT, CandidateT]):
    @property
    def initial_state(self) -> StateT: ...

    def is_terminal(self, state: StateT) -> bool: ...

    def propose(self, state: StateT, step_index: int, seeds: SeedStream) -> Sequence[ProposalT]: ...

    def evaluate(self, state: StateT, proposals: Sequence[ProposalT], step_index: int,
                 seeds: SeedStream) -> Sequence[StepwiseCandidate[CandidateT]]: ...

    def advance(self, state: StateT, selected: CandidateT, step_index: int) -> StateT: ...


def normalize_log_weights(log_weights: Sequence[float]) -> tuple[float, ...]:
    """Probabilities proportional to exp(log_weights)."""
    return normalize_smc_log_weights(log_weights)[0]


def categorical_index_from_uniform(probabilities: Sequence[float], uniform: float) -> int:
    """Inverse-CDF draw: the number of cumulative masses that do not exceed ``uniform``."""
    p = np.asarray(probabilities, dtype=np.float64)
    if p.ndim != 1 or p.size == 0:
        raise ValueError("a categorical draw needs a non-empty probability vector")
    if not np.isfinite(p).all() or (p < 0).any() or not p.sum() > 0:
        raise ValueError("categorical probabilities must be finite, non-negative and not all zero")
    if not (np.isfinite(uniform) and 0.0 <= uniform < 1.0):
        raise ValueError("the categorical uniform must lie in [0, 1)")
    cdf = np.cumsum(p / p.sum())
    cdf[-1] = 1.0
    return int(np.count_nonzero(cdf <= uniform))


def select_stepwise_candidate(*, state, candidates, step_index: int, rng: np.random.Generator) -> StepwiseSelection:
    pool = tuple(candidates)
    probabilities = normalize_log_weights([c.log_weight for c in pool])
    chosen = categorical_index_from_uniform(probabilities, float(rng.random()))
    return StepwiseSelection(step_index, state, pool, probabilities, chosen)


class StepwiseSampler:
    """Drives one backend through propose -> evaluate -> select -> advance steps."""

    def __init__(self, backend, seeds: SeedStream, namespace: Sequence[object] = ("stepwise",)):
        self.backend = backend
        self.seeds = seeds
        self.namespace = tuple(namespace)

    def step(self, state, step_index: int) -> StepwiseSelection:
        b = self.backend
        if b.is_terminal(state):
            raise ValueError("the state is terminal; there is no further step")
        proposals = tuple(b.propose(state, step_index, self.seeds))
        if not proposals:
            raise RuntimeError("the backend proposed nothing for a non-terminal state")
        scored = tuple(b.evaluate(state, proposals, step_index, self.seeds))
        if len(scored) != len(proposals):
            raise RuntimeError(f"the backend scored {len(scored)} candidates for {len(proposals)} proposals")
        rng = self.seeds.generator(*self.namespace, step_index, "select")
        return select_stepwise_candidate(state=state, candidates=scored, step_index=step_index, rng=rng)

    def run(self) -> StepwiseGenerationResult:
        state = self.backend.initial_state
        history: list[StepwiseSelection] = []
        while not self.backend.is_terminal(state):
            chosen = self.step(state, len(history))
            state = self.backend.advance(state, chosen.selected.value, len(history))
            history.append(chosen)
        return StepwiseGenerationResult(state, tuple(history))


def stepwise_generation_step(backend, state, step_index: int, seeds: SeedStream, *,
                             selection_namespace: Sequence[object] = ("stepwise",)) -> StepwiseSelection:
    return StepwiseSampler(backend, seeds, selection_namespace).step(state, step_index)


def run_stepwise_generation(backend, seeds: SeedStream, *,
                            selection_namespace: Sequence[object] = ("stepwise",)) -> StepwiseGenerationResult:
    return StepwiseSampler(backend, seeds, selection_namespace).run()
