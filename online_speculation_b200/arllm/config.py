"""Validated sampling and algorithm configurations for autoregressive models.

Field names, defaults, validation and ``policy_id`` strings follow the
reference (src/inference_scaling/arllm/config.py:18-325) so that configs and
cached artefacts keyed by policy identity carry over.
"""

from __future__ import annotations

from dataclasses import dataclass

from ..shared.config import canonical_float, require_finite, require_positive, require_probability

DEFAULT_MAX_NEW_TOKENS = 32768


@dataclass(frozen=True, slots=True)
class SamplingConfig:
    """The complete stochastic policy of one autoregressive request."""

    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int | None = None
    eos_token_id: int | None = None

    def __post_init__(self) -> None:
        require_positive("temperature", self.temperature)
        require_probability("top_p", self.top_p, include_zero=False)
        if self.top_k is not None:
            require_positive("top_k", self.top_k)
        if self.eos_token_id is not None and self.eos_token_id < 0:
            raise ValueError("eos_token_id must be non-negative")

    @property
    def policy_id(self) -> str:
        return (f"temperature={canonical_float(self.temperature)};top_p={canonical_float(self.top_p)};"
                f"top_k={self.top_k};eos={self.eos_token_id}")

    @property
    def full_support(self) -> bool:
        return self.top_k is None and self.top_p >= 1


def _check_schedule(name: str) -> None:
    if name not in ("uniform", "inverse_length", "multiscale"):
        raise ValueError("unknown MH suffix_schedule")


@dataclass(frozen=True, slots=True)
class MHConfig:
    """Staged suffix MH for the power target p^alpha."""

    alpha: float = 4.0
    total_length: int = DEFAULT_MAX_NEW_TOKENS
    block_size: int = 32
    steps_per_block: int = 10
    chains: int = 1
    suffix_schedule: str = "uniform"
    iterations: int | None = None

    def __post_init__(self) -> None:
        require_finite("alpha", self.alpha)
        if self.alpha < 1:
            raise ValueError("alpha must be at least one")
        for name in ("total_length", "block_size", "steps_per_block", "chains"):
            require_positive(name, getattr(self, name))
        if self.block_size > self.total_length:
            raise ValueError("block_size cannot exceed total_length")
        _check_schedule(self.suffix_schedule)
        if self.iterations is not None:
            require_positive("iterations", self.iterations)

    @property
    def stages(self) -> tuple[int, ...]:
        if self.iterations is not None:
            return (self.total_length,)
        lengths = tuple(range(self.block_size, self.total_length + 1, self.block_size))
        return lengths if lengths and lengths[-1] == self.total_length else (*lengths, self.total_length)

    @property
    def stage_updates(self) -> int:
        return self.steps_per_block if self.iterations is None else self.iterations

    @property
    def proposal(self) -> SamplingConfig:
        """The full-support proposal at temperature 1 / alpha."""
        return SamplingConfig(temperature=1.0 / self.alpha)


@dataclass(frozen=True, slots=True)
class RewardMHConfig:
    """Full-sequence MH budget for p(y) exp(r(y) / tau)."""

    total_length: int = DEFAULT_MAX_NEW_TOKENS
    block_size: int = 32
    steps_per_block: int = 10
    reward_temperature: float = 0.1
    suffix_schedule: str = "uniform"
    iterations: int | None = None

    def __post_init__(self) -> None:
        for name in ("total_length", "block_size", "steps_per_block"):
            require_positive(name, getattr(self, name))
        require_positive("reward_temperature", self.reward_temperature)
        if self.block_size > self.total_length:
            raise ValueError("block_size cannot exceed total_length")
        _check_schedule(self.suffix_schedule)
        if self.iterations is not None:
            require_positive("iterations", self.iterations)

    @property
    def updates(self) -> int:
        if self.iterations is not None:
            return self.iterations
        return -(-self.total_length // self.block_size) * self.steps_per_block


@dataclass(frozen=True, slots=True)
class ConditionalISConfig:
    candidate_count: int = 4
    rollout_count: int = 4
    block_size: int = 16
    total_length: int = DEFAULT_MAX_NEW_TOKENS
    reward_temperature: float = 1.0
    importance_log_ratio_clip: float | None = None
    apply_importance_correction: bool = True
    rollout_design: str = "iid"
    exact_rollout_early_stop: bool = False
    rollout_log_weight_bounds: tuple[float, float] | None = None
    rollout_evaluation_batch_size: int = 1

    def __post_init__(self) -> None:
        for name in ("candidate_count", "rollout_count", "block_size", "total_length"):
            require_positive(name, getattr(self, name))
        require_positive("reward_temperature", self.reward_temperature)
        if self.importance_log_ratio_clip is not None:
            require_positive("importance_log_ratio_clip", self.importance_log_ratio_clip)
            if not self.apply_importance_correction:
                raise ValueError("importance_log_ratio_clip requires apply_importance_correction=True")
        if self.block_size > self.total_length:
            raise ValueError("block_size cannot exceed total_length")
        if self.rollout_design not in ("iid", "sobol", "lattice"):
            raise ValueError("rollout_design must be iid, sobol or lattice")
        if self.exact_rollout_early_stop and self.rollout_log_weight_bounds is None:
            raise ValueError("exact early stopping needs rollout_log_weight_bounds")
        if self.rollout_log_weight_bounds is not None:
            lo, hi = self.rollout_log_weight_bounds
            require_finite("lower log-weight bound", lo)
            require_finite("upper log-weight bound", hi)
            if lo > hi:
                raise ValueError("rollout_log_weight_bounds must be ordered")
        require_positive("rollout_evaluation_batch_size", self.rollout_evaluation_batch_size)
