"""Validation helpers and runtime configuration shared by every model family.

Mirrors the validators and canonical policy-identity formatting of the
reference (src/inference_scaling/shared/config.py:9-97): a policy parameter is
identified by ``repr(float(value))`` so that identity strings round-trip.
"""

from __future__ import annotations

from dataclasses import dataclass
from math import isfinite


def canonical_float(value: float) -> str:
    number = float(value)
    if not isfinite(number):
        raise ValueError(f"a policy parameter must be finite, got {value!r}")
    return repr(number)


def require_finite(name: str, value) -> None:
    if not isfinite(float(value)):
        raise ValueError(f"{name} must be finite, got {value!r}")


def require_positive(name: str, value) -> None:
    require_finite(name, value)
    if value <= 0:
        raise ValueError(f"{name} must be positive, got {value!r}")


def require_nonnegative(name: str, value) -> None:
    require_finite(name, value)
    if value < 0:
        raise ValueError(f"{name} must be non-negative, got {value!r}")


def require_probability(name: str, value: float, *, include_zero: bool = True) -> None:
    require_finite(name, value)
    low_ok = value >= 0 if include_zero else value > 0
    if not low_ok or value > 1:
        raise ValueError(f"{name} must lie in {'[0, 1]' if include_zero else '(0, 1]'}, got {value!r}")


@dataclass(frozen=True, slots=True)
class RuntimeConfig:
    seed: int = 0
    max_batch_size: int = 32
    max_batch_tokens: int = 4096
    deterministic: bool = True

    def __post_init__(self) -> None:
        require_nonnegative("seed", self.seed)
        require_positive("max_batch_size", self.max_batch_size)
        require_positive("max_batch_tokens", self.max_batch_tokens)


@dataclass(frozen=True, slots=True)
class SMCForestConfig:
    particle_count: int = 8
    branch_factor: int = 2
    rollout_count: int = 4
    block_size: int = 16
    total_length: int = 128
    reward_temperature: float = 1.0
    reward_workers: int = 4
    reuse_rollout_forest: bool = True

    def __post_init__(self) -> None:
        for name in ("particle_count", "branch_factor", "rollout_count", "block_size", "total_length",
                     "reward_temperature", "reward_workers"):
            require_positive(name, getattr(self, name))
        if self.block_size > self.total_length:
            raise ValueError("block_size cannot exceed total_length")
