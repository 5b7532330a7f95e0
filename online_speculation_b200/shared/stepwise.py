"""Generic propose -> evaluate -> select -> advance loop over opaque states
(sequential importance resampling with one candidate kept per step).

Reference: src/inference_scaling/shared/stepwise.py:67-214.  Selection draws
one explicit uniform from the stream ``(namespace..., step, "select")``.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import isfinite
from typing import Generic, Protocol, TypeVar, runtime_checkable

import numpy as np

from .rng import SeedStream

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
    if not len(log_weights):
        raise ValueError("at least one candidate log-weight is required")
    v = np.asarray(log_weights, dtype=np.float64)
    if not np.all(np.isfinite(v)):
        raise ValueError("candidate log-weights must be finite")
    w = np.exp(v - v.max())
    total = float(w.sum())
    if not isfinite(total) or total <= 0:
        raise ValueError("candidate weights cannot be normalized")
    return tuple(float(x) for x in w / total)


def categorical_index_from_uniform(probabilities: Sequence[float], uniform: float) -> int:
    p = np.asarray(probabilities, dtype=np.float64)
    if p.ndim != 1 or not len(p):
        raise ValueError("categorical probabilities must be a non-empty vector")
    if not np.all(np.isfinite(p)) or np.any(p < 0):
        raise ValueError("categorical probabilities must be finite and non-negative")
    total = float(p.sum())
    if not isfinite(total) or total <= 0:
        raise ValueError("categorical probabilities must have positive mass")
    if not isfinite(uniform) or not 0.0 <= uniform < 1.0:
        raise ValueError("uniform must be finite and lie in [0, 1)")
    cdf = np.cumsum(p / total)
    cdf[-1] = 1.0
    return int(np.searchsorted(cdf, uniform, side="right"))


def select_stepwise_candidate(*, state, candidates, step_index: int, rng: np.random.Generator) -> StepwiseSelection:
    evaluated = tuple(candidates)
    probs = normalize_log_weights([c.log_weight for c in evaluated])
    return StepwiseSelection(step_index, state, evaluated, probs, categorical_index_from_uniform(probs, float(rng.random())))


def stepwise_generation_step(backend, state, step_index: int, seeds: SeedStream, *,
                             selection_namespace: Sequence[object] = ("stepwise",)) -> StepwiseSelection:
    if backend.is_terminal(state):
        raise ValueError("cannot advance a terminal generation state")
    proposals = tuple(backend.propose(state, step_index, seeds))
    if not proposals:
        raise RuntimeError("stepwise backend returned no candidates")
    candidates = tuple(backend.evaluate(state, proposals, step_index, seeds))
    if len(candidates) != len(proposals):
        raise RuntimeError("stepwise backend must evaluate every proposal exactly once")
    return select_stepwise_candidate(state=state, candidates=candidates, step_index=step_index,
                                     rng=seeds.generator(*selection_namespace, step_index, "select"))


def run_stepwise_generation(backend, seeds: SeedStream, *,
                            selection_namespace: Sequence[object] = ("stepwise",)) -> StepwiseGenerationResult:
    state = backend.initial_state
    steps = []
    index = 0
    while not backend.is_terminal(state):
        sel = stepwise_generation_step(backend, state, index, seeds, selection_namespace=selection_namespace)
        state = backend.advance(state, sel.selected.value, index)
        steps.append(sel)
        index += 1
    return StepwiseGenerationResult(state, tuple(steps))
