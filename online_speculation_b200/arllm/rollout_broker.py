"""Resumable partial rollouts and an over-provisioning rollout broker.

State is token sequences, not engine KV objects, so an interrupted rollout can
resume on any backend (and survives cache eviction).  Each resumed segment is
sampled from the requested policy given the tokens so far; the log-probabilities
returned are those actually used.  ``AsyncRolloutBroker.run_until`` advances
requests in ``chunk_tokens`` segments (partial trajectories first, then by
priority) until ``completion_target`` of them finished, bounding the work left
unfinished in an over-provisioned batch.

Reference behaviour: src/inference_scaling/arllm/rollout_broker.py:32-333.
"""

from __future__ import annotations

import threading
from collections.abc import Callable, Sequence
from dataclasses import dataclass

from ..shared.rng import SeedStream
from ..shared.types import TokenSequence
from .acceleration import sample_batch_with_callback
from .types import AutoregressiveBackend, GenerationRequest, SequenceSample


@dataclass(frozen=True, slots=True)
class PartialRollout:
    request: GenerationRequest
    token_ids: TokenSequence = ()
    token_logprobs: tuple[float, ...] = ()
    reference_token_logprobs: tuple[float, ...] | None = None
    reference_policy_id: str | None = None
    policy_id: str | None = None
    model_id: str | None = None
    finish_reason: str = "partial"
    segments: int = 0
    priority: float = 0.0

    def __post_init__(self) -> None:
        if len(self.token_ids) != len(self.token_logprobs):
            raise ValueError("partial rollout tokens and log-probabilities must align")
        if (self.reference_token_logprobs is None) != (self.reference_policy_id is None):
            raise ValueError("partial reference probabilities require a policy id")
        if self.reference_token_logprobs is not None and len(self.reference_token_logprobs) != len(self.token_ids):
            raise ValueError("partial reference probabilities must align with tokens")
        if len(self.token_ids) > self.request.max_new_tokens:
            raise ValueError("partial rollout exceeds its original token budget")
        if self.segments < 0:
            raise ValueError("partial rollout segment count must be non-negative")

    @classmethod
    def from_request(cls, request: GenerationRequest, *, priority: float = 0.0) -> "PartialRollout":
        return cls(request=request, priority=float(priority))

    @property
    def remaining_tokens(self) -> int:
        return self.request.max_new_tokens - len(self.token_ids)

    @property
    def complete(self) -> bool:
        return self.finish_reason != "partial"

    def next_request(self, chunk_tokens: int) -> GenerationRequest:
        if self.complete or self.remaining_tokens <= 0:
            raise ValueError("completed rollout cannot be resumed")
        if chunk_tokens <= 0:
            raise ValueError("chunk_tokens must be positive")
        n = min(int(chunk_tokens), self.remaining_tokens)
        r = self.request
        seed = r.seed if self.segments == 0 else SeedStream(r.seed).derive("partial-rollout", r.request_id,
                                                                             self.segments)
        done = len(self.token_ids)
        return GenerationRequest(r.prefix + self.token_ids, n, r.sampling, seed, f"{r.request_id}:segment:{self.segments}",
                                 r.uniforms[done:done + n] if r.uniforms is not None else None)

    def append(self, segment: GenerationRequest, sample: SequenceSample) -> "PartialRollout":
        want = self.request.prefix + self.token_ids
        if segment.prefix != want or sample.prefix != want:
            raise RuntimeError("partial rollout segment has the wrong prefix")
        if sample.request_id != segment.request_id:
            raise RuntimeError("partial rollout segment has the wrong request id")
        if sample.policy_id != self.request.sampling.policy_id:
            raise RuntimeError("partial rollout segment used the wrong policy")
        if len(sample.token_ids) > segment.max_new_tokens:
            raise RuntimeError("partial rollout segment exceeded its chunk budget")
        if not sample.token_ids and self.remaining_tokens:
            raise RuntimeError("partial rollout segment made no progress")
        if self.model_id is not None and sample.model_id != self.model_id:
            raise RuntimeError("partial rollout changed model between segments")
        if self.reference_policy_id is not None:
            if sample.reference_policy_id != self.reference_policy_id or sample.reference_token_logprobs is None:
                raise RuntimeError("partial rollout changed or dropped its reference policy between segments")
        elif self.segments and sample.reference_policy_id is not None:
            raise RuntimeError("partial rollout added reference scores after the first segment")
        toks = self.token_ids + sample.token_ids
        if sample.reference_token_logprobs is None:
            refs, ref_id = None, None
        else:
            refs, ref_id = (self.reference_token_logprobs or ()) + sample.reference_token_logprobs, \
                sample.reference_policy_id
        finished = sample.finish_reason == "eos" or len(toks) >= self.request.max_new_tokens
        reason = "eos" if sample.finish_reason == "eos" else ("length" if finished else "partial")
        return PartialRollout(self.request, toks, self.token_logprobs + sample.token_logprobs, refs, ref_id,
                              sample.policy_id, sample.model_id, reason, self.segments + 1, self.priority)

    def to_sample(self) -> SequenceSample:
        if not self.complete:
            raise ValueError("unfinished rollout cannot be materialized as a sample")
        return SequenceSample(self.request.prefix, self.token_ids, self.token_logprobs, self.policy_id, self.model_id,
                              self.request.request_id, self.finish_reason, self.reference_token_logprobs,
                              self.reference_policy_id)


@dataclass(frozen=True, slots=True)
class RolloutBrokerSnapshot:
    requested_completion_target: int
    completed_rollouts: int
    partial_rollouts: int
    completion_overshoot: int
    physical_batches: int
    sampled_segments: int
    generated_tokens: int
    initial_partial_tokens: int
    partial_tokens_preserved: int
    resumed_prefill_tokens: int


@dataclass(frozen=True, slots=True)
class RolloutBrokerResult:
    completed: tuple[SequenceSample, ...]
    partial: tuple[PartialRollout, ...]
    snapshot: RolloutBrokerSnapshot


class AsyncRolloutBroker:
    def __init__(self, backend: AutoregressiveBackend, *, chunk_tokens: int = 16, max_batch_size: int | None = None):
        if chunk_tokens <= 0:
            raise ValueError("chunk_tokens must be positive")
        if max_batch_size is not None and max_batch_size <= 0:
            raise ValueError("max_batch_size must be positive")
        self.backend, self.chunk_tokens, self.max_batch_size = backend, int(chunk_tokens), max_batch_size

    def run_until(self, rollouts: Sequence[PartialRollout | GenerationRequest], *,
                  completion_target: int | None = None,
                  on_complete: Callable[[SequenceSample], None] | None = None,
                  on_segment: Callable[[PartialRollout], None] | None = None) -> RolloutBrokerResult:
        states = [x if isinstance(x, PartialRollout) else PartialRollout.from_request(x) for x in rollouts]
        if not states:
            if completion_target not in (None, 0):
                raise ValueError("an empty broker run cannot complete requests")
            target = 0
        else:
            target = len(states) if completion_target is None else int(completion_target)
            if not 0 < target <= len(states):
                raise ValueError("completion_target must lie within the submitted rollout count")
        ids = [s.request.request_id for s in states]
        if len(ids) != len(set(ids)):
            raise ValueError("rollout broker request ids must be unique")
        if any(s.complete for s in states):
            raise ValueError("completed samples should not be resubmitted to the broker")
        init_partial = sum(len(s.token_ids) for s in states)
        done: list[SequenceSample] = []
        pending = list(states)
        batches = segs = gen = resumed = 0
        while pending and len(done) < target:
            pending.sort(key=lambda s: (-s.priority, -int(bool(s.token_ids)), -len(s.token_ids), s.request.request_id))
            n = self.max_batch_size or len(pending)
            batch, pending = pending[:n], pending[n:]
            reqs = [s.next_request(self.chunk_tokens) for s in batch]
            order: list[int] = []
            lock = threading.Lock()

            def finished(i, _s, order=order, lock=lock):
                with lock:
                    order.append(i)

            got = sample_batch_with_callback(self.backend, reqs, finished)
            if len(got) != len(batch):
                raise RuntimeError("rollout backend returned an invalid segment count")
            order += [i for i in range(len(got)) if i not in order]
            batches += 1
            segs += len(got)
            gen += sum(len(s.token_ids) for s in got)
            resumed += sum(len(s.token_ids) for s in batch)
            seen = set()
            for i in order:
                if i in seen:
                    continue
                seen.add(i)
                st = batch[i].append(reqs[i], got[i])
                if on_segment is not None:
                    on_segment(st)
                if st.complete:
                    smp = st.to_sample()
                    done.append(smp)
                    if on_complete is not None:
                        on_complete(smp)
                else:
                    pending.append(st)
        snap = RolloutBrokerSnapshot(target, len(done), len(pending), max(0, len(done) - target), batches, segs, gen,
                                     init_partial, sum(len(s.token_ids) for s in pending), resumed)
        return RolloutBrokerResult(tuple(done), tuple(pending), snap)


__all__ = ["AsyncRolloutBroker", "PartialRollout", "RolloutBrokerResult", "RolloutBrokerSnapshot"]
