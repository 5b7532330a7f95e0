"""Attach model metadata (tokenizer, statistics, snapshots) to a probability-preserving executor.

Reference behaviour: src/inference_scaling/arllm/backends/execution.py.
"""

from __future__ import annotations

from typing import Any


class ExecutionBackend:
    def __init__(self, executor: Any, backend: Any):
        self.executor, self.backend = executor, backend

    @property
    def model_id(self):
        return self.executor.model_id

    @property
    def tokenizer(self):
        return self.backend.tokenizer

    @property
    def parameter_count(self):
        return self.backend.parameter_count

    def sample_batch(self, requests):
        return self.executor.sample_batch(requests)

    def score_batch(self, requests):
        return self.executor.score_batch(requests)

    def score_statistics_batch(self, requests, *, confidence_top_k=None):
        return self.backend.score_statistics_batch(requests, confidence_top_k=confidence_top_k)

    def encode(self, text, *, add_special_tokens=True):
        return self.backend.encode(text, add_special_tokens=add_special_tokens)

    def decode(self, tokens, *, skip_special_tokens=True):
        return self.backend.decode(tokens) if skip_special_tokens else self.backend.decode(
            tokens, skip_special_tokens=False)

    def snapshot(self):
        return self.backend.snapshot()


def execution_model(executor: Any) -> Any:
    """The first object below cache / batching wrappers that exposes a tokenizer."""
    seen = set()
    while executor is not None and id(executor) not in seen:
        seen.add(id(executor))
        if hasattr(executor, "tokenizer"):
            return executor
        executor = getattr(executor, "backend", getattr(executor, "_backend", None))
    raise ValueError("execution wrapper does not expose model/tokenizer metadata")


__all__ = ["ExecutionBackend", "execution_model"]
