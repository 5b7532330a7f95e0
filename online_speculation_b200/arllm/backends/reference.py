"""Rescales temperatures so that an outer temperature of 1 means the wrapped backend's
reference temperature T_ref.

MH kernels written against "temperature 1 is the base policy" then target the same
base law as an IS run at T_ref.  Log-probabilities are the model's own; only policy
and model ids are rewritten into the outer contract, and the reference (base-policy)
log-probabilities are passed through when the inner sample carries them under the
scaled base policy.  Model-id suffix and policy translation follow
src/inference_scaling/arllm/backends/reference.py (cache identity).
"""

from __future__ import annotations

from dataclasses import replace
from math import isfinite

from ..config import SamplingConfig


class ReferencePolicyBackend:
    def __init__(self, backend, *, temperature: float):
        if not (isfinite(temperature) and temperature > 0):
            raise ValueError(f"the reference temperature has to be a positive number, not {temperature!r}")
        self.backend = backend
        self.temperature = temperature
        self.model_id = f"{backend.model_id}|reference-temperature={temperature}"

    def _inner(self, sampling: SamplingConfig | None) -> SamplingConfig:
        outer = sampling if sampling is not None else SamplingConfig()
        return replace(outer, temperature=outer.temperature * self.temperature)

    def _reference_logprobs(self, sample, eos):
        base_inner = self._inner(SamplingConfig(eos_token_id=eos)).policy_id
        if sample.policy_id == base_inner:
            return sample.token_logprobs
        if sample.reference_policy_id == base_inner:
            return sample.reference_token_logprobs
        return None

    def sample_batch(self, requests):
        inner_requests = [replace(r, sampling=self._inner(r.sampling)) for r in requests]
        samples = self.backend.sample_batch(inner_requests)
        if len(samples) != len(requests):
            raise RuntimeError(f"the wrapped backend returned {len(samples)} samples for {len(requests)} requests")
        translated = []
        for outer, inner, sample in zip(requests, inner_requests, samples):
            if sample.model_id != self.backend.model_id or sample.policy_id != inner.sampling.policy_id:
                raise RuntimeError("the wrapped backend answered under another model or policy")
            eos = outer.sampling.eos_token_id
            reference = self._reference_logprobs(sample, eos)
            translated.append(replace(
                sample, model_id=self.model_id, policy_id=outer.sampling.policy_id,
                reference_token_logprobs=reference,
                reference_policy_id=SamplingConfig(eos_token_id=eos).policy_id if reference is not None else None))
        return translated

    def score_batch(self, requests):
        return self.backend.score_batch([replace(r, sampling=self._inner(r.sampling)) for r in requests])


__all__ = ["ReferencePolicyBackend"]
