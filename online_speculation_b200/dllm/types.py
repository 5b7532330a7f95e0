"""Requests, committed reverse-diffusion traces and the backend contract for dLLMs.

Field names and validation follow src/inference_scaling/dllm/types.py:14-125
(the algorithm/backend contract).
"""

from __future__ import annotations

from dataclasses import dataclass
from math import isclose, isfinite
from typing import Protocol, Sequence, runtime_checkable

from ..shared.types import TokenSequence
from .config import DiffusionSamplingConfig


@dataclass(frozen=True, slots=True)
class DiffusionGenerationRequest:
    prefix: TokenSequence
    generation_length: int
    sampling: DiffusionSamplingConfig
    seed: int
    request_id: str

    def __post_init__(self) -> None:
        self.sampling.validate_generation_length(self.generation_length, prefix_length=len(self.prefix))
        if self.seed < 0:
            raise ValueError("seed must be non-negative")


@dataclass(frozen=True, slots=True)
class DiffusionTraceStep:
    """One committed transition; positions are relative to the continuation.

    ``logprob`` holds the selected tokens' log-probabilities plus, for random
    remasking, the log-probability of the uniformly drawn position subset.
    """

    block_index: int
    step_index: int
    positions: tuple[int, ...]
    token_ids: TokenSequence
    logprob: float | None

    def __post_init__(self) -> None:
        if self.block_index < 0 or self.step_index < 0:
            raise ValueError("trace indices must be non-negative")
        if len(self.positions) != len(self.token_ids):
            raise ValueError("each committed position must have one token")
        if any(b <= a for a, b in zip(self.positions, self.positions[1:])):
            raise ValueError("committed positions must be strictly sorted")
        if self.logprob is not None and not isfinite(self.logprob):
            raise ValueError("trace log-probability must be finite")


@dataclass(frozen=True, slots=True)
class DiffusionSample:
    prefix: TokenSequence
    token_ids: TokenSequence
    trace: tuple[DiffusionTraceStep, ...]
    trajectory_logprob: float | None
    policy_id: str
    model_id: str
    request_id: str
    finish_reason: str = "length"

    def __post_init__(self) -> None:
        seen: set[int] = set()
        for step in self.trace:
            for pos, tok in zip(step.positions, step.token_ids):
                if not 0 <= pos < len(self.token_ids):
                    raise ValueError("trace position lies outside the continuation")
                if pos in seen:
                    raise ValueError("a continuation position was committed more than once")
                if self.token_ids[pos] != tok:
                    raise ValueError("trace token does not match the final continuation")
                seen.add(pos)
        if self.trace and len(seen) != len(self.token_ids):
            raise ValueError("a complete trace must commit every continuation position")
        if self.trajectory_logprob is not None:
            if self.token_ids and not self.trace:
                raise ValueError("an exact trajectory requires a complete trace")
            if not isfinite(self.trajectory_logprob):
                raise ValueError("trajectory_logprob must be finite")
            if any(s.logprob is None for s in self.trace):
                raise ValueError("an exact trajectory requires every step probability")
            total = sum(float(s.logprob) for s in self.trace)
            if not isclose(total, self.trajectory_logprob, rel_tol=1e-9, abs_tol=1e-9):
                raise ValueError("trajectory_logprob must equal the sum of step log-probabilities")

    @property
    def full_sequence(self) -> TokenSequence:
        return self.prefix + self.token_ids


@dataclass(frozen=True, slots=True)
class DiffusionTrajectoryScoreRequest:
    sample: DiffusionSample
    sampling: DiffusionSamplingConfig


@runtime_checkable
class DiffusionBackend(Protocol):
    @property
    def model_id(self) -> str: ...

    def sample_batch(self, requests: Sequence[DiffusionGenerationRequest]) -> list[DiffusionSample]: ...

    def score_trajectories(self, requests: Sequence[DiffusionTrajectoryScoreRequest]) -> list[float]: ...


__all__ = ["DiffusionBackend", "DiffusionGenerationRequest", "DiffusionSample", "DiffusionTraceStep",
           "DiffusionTrajectoryScoreRequest"]
