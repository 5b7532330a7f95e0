"""Resumable rollouts and a broker that stops once enough of them have finished.

A :class:`PartialRollout` stores tokens, not engine KV state, so an interrupted
rollout can continue on any backend.  Each resumed segment is sampled from the
request's own policy given the tokens so far, and the log-probabilities kept are
the ones that segment actually used.  :class:`AsyncRolloutBroker` advances rollouts
``chunk_tokens`` at a time, most urgent first (priority, then those already
started, then the longest), until ``completion_target`` of them have finished; what
is left is returned as partial rollouts, which bounds the work an
over-provisioned batch wastes.  Segment seeds come from the stream
``(seed, "partial-rollout", request_id, segment)`` and segment request ids end in
``:segment:<n>``, the random-stream and id conventions of
src/inference_scaling/arllm/rollout_broker.py.
"""

from __future__ import annotations

import heapq
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
        n = len(self.token_ids)
        problems = []
        if len(self.token_logprobs) != n:
            problems.append("one log-probability per token")
        if (self.reference_token_logprobs is None) != (self.reference_policy_id is None):
            problems.append("reference log-probabilities and their policy id go together")
        if self.reference_token_logprobs is not None and len(self.reference_token_logprobs) != n:
            problems.append("one reference log-probability per token")
        if n > self.request.max_new_tokens:
            problems.append("no more tokens than the request's budget")
        if self.segments < 0:
            problems.append("a non-negative segment count")
        if problems:
            raise ValueError("inconsistent partial rollout, expected " + "; ".join(problems))

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
            raise ValueError("this rollout is finished; there is nothing to resume")
        if chunk_tokens < 1:
            raise ValueError("chunk_tokens has to be positive")
        r = self.request
        size = min(int(chunk_tokens), self.remaining_tokens)
        offset = len(self.token_ids)
        seed = r.seed if self.segments == 0 else SeedStream(r.seed).derive("partial-rollout", r.request_id,
                                                                             self.segments)
        uniforms = None if r.uniforms is None else r.uniforms[offset:offset + size]
        return GenerationRequest(r.prefix + tuple(self.token_ids), size, r.sampling, seed,
                                 f"{r.request_id}:segment:{self.segments}", uniforms)

    def _segment_problem(self, segment: GenerationRequest, sample: SequenceSample) -> str | None:
        expected = self.request.prefix + tuple(self.token_ids)
        rules = (
            (segment.prefix == expected and sample.prefix == expected, "the segment continues a different prefix"),
            (sample.request_id == segment.request_id, "the sample answers another request"),
            (sample.policy_id == self.request.sampling.policy_id, "the segment used another policy"),
            (len(sample.token_ids) <= segment.max_new_tokens, "the segment exceeded its chunk"),
            (bool(sample.token_ids) or not self.remaining_tokens, "the segment made no progress"),
            (self.model_id is None or sample.model_id == self.model_id, "the model changed between segments"),
            (self.reference_policy_id is None or (sample.reference_policy_id == self.reference_policy_id
                                                  and sample.reference_token_logprobs is not None),
             "the reference policy changed or disappeared between segments"),
            (self.reference_policy_id is not None or not self.segments or sample.reference_policy_id is None,
             "reference scores appeared after the first segment"),
        )
        return next((message for ok, message in rules if not ok), None)

    def append(self, segment: GenerationRequest, sample: SequenceSample) -> "PartialRollout":
        problem = self._segment_problem(segment, sample)
        if problem is not None:
            raise RuntimeError(f"rollout {self.request.request_id!r}: {problem}")
        tokens = tuple(self.token_ids) + tuple(sample.token_ids)
        if sample.reference_token_logprobs is None:
            reference, reference_id = None, None
        else:
            reference = tuple(self.reference_token_logprobs or ()) + tuple(sample.reference_token_logprobs)
            reference_id = sample.reference_policy_id
        if sample.finish_reason == "eos":
            reason = "eos"
        else:
            reason = "length" if len(tokens) >= self.request.max_new_tokens else "partial"
        return PartialRollout(self.request, tokens, tuple(self.token_logprobs) + tuple(sample.token_logprobs),
                              reference, reference_id, sample.policy_id, sample.model_id, reason, self.segments + 1,
                              self.priority)

    def to_sample(self) -> SequenceSample:
        if not self.complete:
            raise ValueError("an unfinished rollout is not a sample yet")
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


def _urgency(r: PartialRollout) -> tuple:
    """Heap key: higher priority, started rollouts, longer rollouts first; request id breaks ties."""
    return (-r.priority, -int(bool(r.token_ids)), -len(r.token_ids), r.request.request_id)


class AsyncRolloutBroker:
    def __init__(self, backend: AutoregressiveBackend, *, chunk_tokens: int = 16, max_batch_size: int | None = None):
        if chunk_tokens < 1:
            raise ValueError("chunk_tokens has to be positive")
        if max_batch_size is not None and max_batch_size < 1:
            raise ValueError("max_batch_size has to be positive")
        self.backend = backend
        self.chunk_tokens = int(chunk_tokens)
        self.max_batch_size = max_batch_size

    @staticmethod
    def _target(count: int, completion_target: int | None) -> int:
        if count == 0:
            if completion_target not in (None, 0):
                raise ValueError("no rollouts were submitted, so none can complete")
            return 0
        target = count if completion_target is None else int(completion_target)
        if not 1 <= target <= count:
            raise ValueError(f"completion_target {target} is outside 1..{count}")
        return target

    def _segment_batch(self, batch: list[PartialRollout]):
        """Sample one segment of every rollout; returns (requests, samples, completion order)."""
        requests = [r.next_request(self.chunk_tokens) for r in batch]
        arrival: list[int] = []
        guard = threading.Lock()

        def on_done(index, _sample):
            with guard:
                if index not in arrival:
                    arrival.append(index)

        samples = sample_batch_with_callback(self.backend, requests, on_done)
        if len(samples) != len(batch):
            raise RuntimeError(f"{len(samples)} segments came back for {len(batch)} rollouts")
        arrival.extend(i for i in range(len(batch)) if i not in arrival)
        return requests, samples, arrival

    def run_until(self, rollouts: Sequence[PartialRollout | GenerationRequest], *,
                  completion_target: int | None = None,
                  on_complete: Callable[[SequenceSample], None] | None = None,
                  on_segment: Callable[[PartialRollout], None] | None = None) -> RolloutBrokerResult:
        states = [r if isinstance(r, PartialRollout) else PartialRollout.from_request(r) for r in rollouts]
        target = self._target(len(states), completion_target)
        ids = [s.request.request_id for s in states]
        if len(set(ids)) != len(ids):
            raise ValueError("rollout request ids have to be distinct")
        if any(s.complete for s in states):
            raise ValueError("finished rollouts cannot be submitted again")
        initial_tokens = sum(len(s.token_ids) for s in states)
        queue = [(_urgency(s), i, s) for i, s in enumerate(states)]
        heapq.heapify(queue)
        tiebreak = len(queue)
        finished: list[SequenceSample] = []
        batches = segments = generated = resumed = 0
        while queue and len(finished) < target:
            width = self.max_batch_size or len(queue)
            batch = [heapq.heappop(queue)[2] for _ in range(min(width, len(queue)))]
            requests, samples, arrival = self._segment_batch(batch)
            batches += 1
            segments += len(samples)
            generated += sum(len(s.token_ids) for s in samples)
            resumed += sum(len(r.token_ids) for r in batch)
            for i in arrival:
                advanced = batch[i].append(requests[i], samples[i])
                if on_segment is not None:
                    on_segment(advanced)
                if advanced.complete:
                    sample = advanced.to_sample()
                    finished.append(sample)
                    if on_complete is not None:
                        on_complete(sample)
                else:
                    heapq.heappush(queue, (_urgency(advanced), tiebreak, advanced))
                    tiebreak += 1
        left = [entry[2] for entry in sorted(queue)]
        snapshot = RolloutBrokerSnapshot(target, len(finished), len(left), max(0, len(finished) - target), batches,
                                         segments, generated, initial_tokens, sum(len(s.token_ids) for s in left),
                                         resumed)
        return RolloutBrokerResult(tuple(finished), tuple(left), snapshot)


__all__ = ["AsyncRolloutBroker", "PartialRollout", "RolloutBrokerResult", "RolloutBrokerSnapshot"]
