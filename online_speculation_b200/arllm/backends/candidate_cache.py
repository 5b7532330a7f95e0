"""Serve frozen candidate samples again by request id; scores still come from a live backend.

A request gets the sample frozen under its own id only when prefix, policy, model and
length budget all agree with it, so a replayed run is the run that was frozen.
Behaviour of src/inference_scaling/arllm/backends/candidate_cache.py.
"""

from __future__ import annotations

from collections.abc import Sequence

from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample


def _mismatch(sample: SequenceSample, request: GenerationRequest, model_id: str) -> str | None:
    checks = (("prefix", sample.prefix == request.prefix),
              ("policy", sample.policy_id == request.sampling.policy_id),
              ("model", sample.model_id == model_id),
              ("length", len(sample.token_ids) <= request.max_new_tokens))
    failed = [name for name, ok in checks if not ok]
    return ", ".join(failed) if failed else None


class CachedCandidateBackend:
    def __init__(self, scoring_backend: AutoregressiveBackend, samples: Sequence[SequenceSample]):
        self.scoring_backend = scoring_backend
        ids = [s.request_id for s in samples]
        if len(set(ids)) != len(ids):
            raise ValueError("frozen candidates must have distinct request ids")
        self.samples = dict(zip(ids, samples))

    @property
    def model_id(self) -> str:
        return self.scoring_backend.model_id

    def _lookup(self, request: GenerationRequest) -> SequenceSample:
        try:
            sample = self.samples[request.request_id]
        except KeyError:
            raise KeyError(f"no frozen candidate for request {request.request_id!r}") from None
        problem = _mismatch(sample, request, self.model_id)
        if problem is not None:
            raise RuntimeError(f"frozen candidate {request.request_id!r} differs from its request in: {problem}")
        return sample

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        return [self._lookup(r) for r in requests]

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        return self.scoring_backend.score_batch(requests)


__all__ = ["CachedCandidateBackend"]
