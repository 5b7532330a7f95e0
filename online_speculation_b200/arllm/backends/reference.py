"""Outer temperature 1 means the configured reference temperature of the wrapped backend.

MH kernels written against "temperature 1 = base policy" then target the same
base law as an IS run at temperature T_ref.  Returned log-probabilities are
the model's own; policy / model ids are translated to the outer contract.
Reference behaviour: src/inference_scaling/arllm/backends/reference.py:11-58.
"""

from __future__ import annotations

from dataclasses import replace
from math import isfinite

from ..config import SamplingConfig


class ReferencePolicyBackend:
    def __init__(self, backend, *, temperature: float):
        if not (isfinite(temperature) and temperature > 0):
            raise ValueError("reference temperature must be finite and positive")
        self.backend, self.temperature = backend, temperature
        self.model_id = f"{backend.model_id}|reference-temperature={temperature}"

    def _policy(self, sampling):
        s = sampling or SamplingConfig()
        return replace(s, temperature=s.temperature * self.temperature)

    def sample_batch(self, requests):
        inner = [replace(r, sampling=self._policy(r.sampling)) for r in requests]
        got = self.backend.sample_batch(inner)
        if len(got) != len(requests):
            raise RuntimeError("reference backend returned an invalid sample count")
        out = []
        for r, ir, s in zip(requests, inner, got):
            if s.model_id != self.backend.model_id or s.policy_id != ir.sampling.policy_id:
                raise RuntimeError("reference backend returned a different sampling policy")
            base = self._policy(SamplingConfig(eos_token_id=r.sampling.eos_token_id))
            if s.policy_id == base.policy_id:
                ref = s.token_logprobs
            elif s.reference_policy_id == base.policy_id:
                ref = s.reference_token_logprobs
            else:
                ref = None
            out.append(replace(s, model_id=self.model_id, policy_id=r.sampling.policy_id,
                               reference_token_logprobs=ref,
                               reference_policy_id=None if ref is None else SamplingConfig(
                                   eos_token_id=r.sampling.eos_token_id).policy_id))
        return out

    def score_batch(self, requests):
        return self.backend.score_batch([replace(r, sampling=self._policy(r.sampling)) for r in requests])


__all__ = ["ReferencePolicyBackend"]
