"""Token and dominant-matmul FLOP accounting (reference: src/inference_scaling/shared/compute.py:10-15)."""

from __future__ import annotations


def dense_forward_flops(parameter_count: int, forward_token_slots: int) -> int:
    """Conventional 2 * parameters * tokens forward estimate."""
    if parameter_count < 0 or forward_token_slots < 0:
        raise ValueError("parameter_count and forward_token_slots must be non-negative")
    return 2 * parameter_count * forward_token_slots


def training_step_flops(parameter_count: int, tokens: int, *, trainable_fraction: float = 1.0,
                        recompute: bool = False) -> int:
    """Forward (2N) + backward (2N for activations + 2N*trainable for weights) per token."""
    passes = 2.0 + 2.0 + 2.0 * trainable_fraction + (2.0 if recompute else 0.0)
    return int(passes * parameter_count * tokens)
