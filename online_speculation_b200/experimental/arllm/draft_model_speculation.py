"""Exact speculative sampling with a separate, smaller draft model.

Each round the draft model proposes k tokens one at a time from its own policy
q (the request's temperature / truncation applied to the draft's
distribution); the target then evaluates all k + 1 positions in ONE forward
(``next_token_probabilities(prefix, block)``, served from its prefix KV cache),
and the standard correction keeps draft token i with probability
min(1, p_i(x) / q_i(x)); at the first rejection it draws from the normalised
residual max(0, p_i - q_i), and after k acceptances it draws one bonus token
from p_{k+1}.  Every emitted token therefore follows the target policy p
exactly; the draft only changes the cost.  Returned log-probabilities are the
target's policy and temperature-1 log-probabilities of the emitted tokens.

Both backends must expose ``next_token_probabilities`` (the engine backend and
the tabular backend do) and share a vocabulary.  Random numbers come from
SeedStream(request.seed), so a request's output does not depend on batching.

Reference behaviour (there through the Transformers assisted-generation loop at
batch size one): src/inference_scaling/experimental/arllm/draft_model_speculation.py:198-507.
"""

from __future__ import annotations

import threading
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from math import log

import numpy as np

from ...arllm.acceleration import DraftModelSpeculationConfig
from ...arllm.backends.tabular import apply_policy
from ...arllm.config import SamplingConfig
from ...arllm.types import GenerationRequest, SequenceSample
from ...shared.rng import SeedStream

SampleCompletionCallback = Callable[[int, SequenceSample], None]


@dataclass(frozen=True, slots=True)
class DraftModelSpeculationSnapshot:
    sample_calls: int
    sampled_sequences: int
    generated_tokens: int
    speculative_requests: int
    speculative_hits: int
    draft_tokens_proposed: int
    draft_tokens_accepted: int
    verification_rounds: int
    draft_model_forward_calls: int
    ordinary_batched_requests: int

    @property
    def draft_acceptance_rate(self) -> float:
        return self.draft_tokens_accepted / self.draft_tokens_proposed if self.draft_tokens_proposed else 0.0

    @property
    def mean_tokens_per_round(self) -> float:
        return self.generated_tokens / self.verification_rounds if self.verification_rounds else 0.0


def _categorical(p: np.ndarray, u: float) -> int:
    c = np.cumsum(p)
    c /= c[-1]
    return min(int(np.searchsorted(c, u, side="right")), len(p) - 1)


class DraftModelSpeculativeBackend:
    def __init__(self, target, draft, *, config: DraftModelSpeculationConfig | None = None):
        if target is draft:
            raise ValueError("target and draft models must be distinct")
        for b in (target, draft):
            if not callable(getattr(b, "next_token_probabilities", None)):
                raise TypeError("both backends must provide next_token_probabilities(prefix, block)")
        tv, dv = getattr(target, "vocab_size", None), getattr(draft, "vocab_size", None)
        if tv is not None and dv is not None and tv != dv:
            raise ValueError("target and draft models must share a vocabulary")
        self.target, self.draft = target, draft
        self.config = config or DraftModelSpeculationConfig()
        self._lock = threading.Lock()
        self._n = dict(sample_calls=0, sampled_sequences=0, generated_tokens=0, speculative_requests=0,
                       speculative_hits=0, draft_tokens_proposed=0, draft_tokens_accepted=0, verification_rounds=0,
                       draft_model_forward_calls=0, ordinary_batched_requests=0)

    @property
    def model_id(self) -> str:
        return self.target.model_id

    @property
    def draft_model_id(self) -> str:
        return self.draft.model_id

    @property
    def parameter_count(self):
        return getattr(self.target, "parameter_count", 1)

    @property
    def draft_parameter_count(self):
        return getattr(self.draft, "parameter_count", 1)

    def _sample_one(self, req: GenerationRequest) -> SequenceSample:
        if req.uniforms is not None or req.arithmetic_uniform is not None:
            raise ValueError("draft-model speculation cannot consume explicit token or arithmetic uniforms")
        pol = req.sampling
        ref = SamplingConfig(eos_token_id=pol.eos_token_id)
        ss = SeedStream(req.seed)
        ctx = tuple(req.prefix)
        toks: list[int] = []
        logq: list[float] = []
        logp: list[float] = []
        finish = "length"
        proposed = accepted = rounds = draft_calls = 0
        rnd = 0
        while len(toks) < req.max_new_tokens and finish == "length":
            k = min(self.config.draft_tokens, req.max_new_tokens - len(toks))
            rng = ss.generator("draft-model-speculation", rnd)
            rnd += 1
            # draft: k sequential proposals from q (each one incremental forward of the draft model)
            block: list[int] = []
            qs: list[np.ndarray] = []
            for _ in range(k):
                q = apply_policy(self.draft.next_token_probabilities(ctx + tuple(block))[-1], pol)
                draft_calls += 1
                t = _categorical(q, float(rng.random()))
                qs.append(q)
                block.append(t)
                if pol.eos_token_id is not None and t == pol.eos_token_id:
                    break
            # target: every position of the block in one forward
            base = self.target.next_token_probabilities(ctx, tuple(block))
            rounds += 1
            proposed += len(block)
            emitted: list[int] = []
            for i, t in enumerate(block):
                p = apply_policy(base[i], pol)
                if float(rng.random()) * qs[i][t] < p[t]:          # accept with min(1, p / q)
                    emitted.append(t)
                    accepted += 1
                    continue
                resid = np.maximum(p - qs[i], 0.0)
                emitted.append(_categorical(resid if resid.sum() > 0 else p, float(rng.random())))
                break
            else:
                # every proposal accepted: one bonus token from the target after the block
                if not (pol.eos_token_id is not None and block and block[-1] == pol.eos_token_id):
                    emitted.append(_categorical(apply_policy(base[len(block)], pol), float(rng.random())))
            for j, t in enumerate(emitted):
                if len(toks) >= req.max_new_tokens:
                    break
                pj = apply_policy(base[j], pol)
                toks.append(int(t))
                logq.append(float(log(pj[t])))
                logp.append(float(log(base[j][t])) if base[j][t] > 0 else float("-inf"))
                ctx = ctx + (int(t),)
                if pol.eos_token_id is not None and t == pol.eos_token_id:
                    finish = "eos"
                    break
        with self._lock:
            n = self._n
            n["speculative_requests"] += 1
            n["speculative_hits"] += int(proposed > 0)
            n["draft_tokens_proposed"] += proposed
            n["draft_tokens_accepted"] += accepted
            n["verification_rounds"] += rounds
            n["draft_model_forward_calls"] += draft_calls
        finite = all(np.isfinite(v) for v in logp)
        return SequenceSample(tuple(req.prefix), tuple(toks), tuple(logq), pol.policy_id, self.target.model_id,
                              req.request_id, finish, tuple(logp) if finite else None,
                              ref.policy_id if finite else None)

    def _sample_batch(self, requests: Sequence[GenerationRequest],
                      on_complete: SampleCompletionCallback | None) -> list[SequenceSample]:
        if not requests:
            return []
        if self.config.single_request_only and len(requests) > 1:
            out = list(self.target.sample_batch(requests))
            with self._lock:
                self._n["ordinary_batched_requests"] += len(requests)
            if on_complete is not None:
                for i, s in enumerate(out):
                    on_complete(i, s)
        else:
            out = []
            for i, r in enumerate(requests):
                s = self._sample_one(r)
                out.append(s)
                if on_complete is not None:
                    on_complete(i, s)
        with self._lock:
            self._n["sample_calls"] += 1
            self._n["sampled_sequences"] += len(out)
            self._n["generated_tokens"] += sum(len(s.token_ids) for s in out)
        return out

    def sample_batch(self, requests) -> list[SequenceSample]:
        return self._sample_batch(tuple(requests), None)

    def sample_batch_with_callback(self, requests, on_complete: SampleCompletionCallback) -> list[SequenceSample]:
        return self._sample_batch(tuple(requests), on_complete)

    def score_batch(self, requests):
        return self.target.score_batch(requests)

    def next_token_probabilities(self, prefix, block=()):
        return self.target.next_token_probabilities(prefix, block)

    def snapshot(self) -> DraftModelSpeculationSnapshot:
        with self._lock:
            return DraftModelSpeculationSnapshot(**self._n)


__all__ = ["DraftModelSpeculationSnapshot", "DraftModelSpeculativeBackend"]
