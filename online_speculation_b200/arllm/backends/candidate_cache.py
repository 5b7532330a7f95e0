"""Replay of frozen candidate samples by request id, with scoring delegated to a live backend.

A request can only retrieve the sample frozen under the same request id,
prefix, policy and model (and no longer than its budget).
Reference behaviour: src/inference_scaling/arllm/backends/candidate_cache.py:15-59.
"""

from __future__ import annotations

from collections.abc import Sequence

from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample


class CachedCandidateBackend:
    def __init__(self, scoring_backend: AutoregressiveBackend, samples: Sequence[SequenceSample]):
        self.scoring_backend = scoring_backend
        self.samples = {s.request_id: s for s in samples}
        if len(self.samples) != len(samples):
            raise ValueError("cached candidate request ids must be unique")

    @property
    def model_id(self) -> str:
        return self.scoring_backend.model_id

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        out = []
        for r in requests:
            s = self.samples.get(r.request_id)
            if s is None:
                raise KeyError(f"candidate request {r.request_id!r} is absent from the frozen cache")
            if (s.prefix != r.prefix or s.policy_id != r.sampling.policy_id or s.model_id != self.model_id
                    or len(s.token_ids) > r.max_new_tokens):
                raise RuntimeError("cached candidate does not match its frozen request")
            out.append(s)
        return out

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        return self.scoring_backend.score_batch(requests)


__all__ = ["CachedCandidateBackend"]
