"""Rollout accelerators that leave the sampled law unchanged.

* :class:`ActiveBatchSpeculationConfig`: how many draft tokens to propose as a
  function of the active batch (speculate only in the latency-bound long tail).
* :class:`RolloutTokenTree`: a bounded table from recent-token contexts to
  next-token counts, filled from finished rollouts.  Its drafts are proposals for
  exact verification: a verifier keeps a draft token only if it equals the token
  the target's own inverse-CDF draw yields at that position, so no draft
  probability ever enters an importance weight.
* :class:`StreamingRewardEvaluator`: reward work for each sequence starts on a
  thread pool as soon as that sequence finishes, overlapping the rest of the batch.
* :class:`LowPriorityRunAheadBackend`: fills the token tree in idle time with
  bounded, preemptible background chunks; a foreground call waits for at most the
  chunk in flight.

Config field names and snapshot fields follow src/inference_scaling/arllm/acceleration.py.
"""

from __future__ import annotations

import queue
import threading
import time
from collections import Counter, OrderedDict
from collections.abc import Callable, Iterable, Sequence
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass
from math import isfinite
from typing import Any

import numpy as np

from ..shared.types import TokenSequence
from .types import AutoregressiveBackend, GenerationRequest, SequenceSample

SampleCompletionCallback = Callable[[int, SequenceSample], None]
TokenReward = Callable[[TokenSequence, TokenSequence], float]


@dataclass(frozen=True, slots=True)
class SpeculationTier:
    """At most ``draft_tokens`` drafts while the active batch holds at most ``max_batch`` requests."""

    max_batch: int
    draft_tokens: int

    def __post_init__(self) -> None:
        if self.max_batch < 1 or self.draft_tokens < 0:
            raise ValueError("a speculation tier needs max_batch >= 1 and draft_tokens >= 0")


@dataclass(frozen=True, slots=True)
class ActiveBatchSpeculationConfig:
    tiers: tuple[SpeculationTier, ...] = (SpeculationTier(4, 8), SpeculationTier(16, 4), SpeculationTier(512, 0))
    min_context_tokens: int = 2
    min_token_probability: float = 0.1
    tree_max_context_tokens: int = 24
    tree_max_contexts: int = 100_000
    vllm_max_cached_requests: int = 10_000
    stochastic_tree: bool = False

    def __post_init__(self) -> None:
        bounds = [t.max_batch for t in self.tiers]
        if not bounds or any(b <= a for a, b in zip(bounds, bounds[1:])):
            raise ValueError("tiers must be non-empty with strictly increasing max_batch")
        if self.min_context_tokens < 1 or self.tree_max_context_tokens < 1 or self.tree_max_contexts < 1:
            raise ValueError("context lengths and the context budget must be positive")
        if not 0.0 <= self.min_token_probability <= 1.0:
            raise ValueError("min_token_probability is a probability")
        if self.vllm_max_cached_requests < 0:
            raise ValueError("vllm_max_cached_requests cannot be negative")

    @property
    def maximum_draft_tokens(self) -> int:
        return max(t.draft_tokens for t in self.tiers)

    def draft_tokens(self, active_batch: int) -> int:
        if active_batch < 1:
            raise ValueError("the active batch holds at least one request")
        bounds = np.asarray([t.max_batch for t in self.tiers])
        tier = min(int(np.searchsorted(bounds, active_batch)), len(self.tiers) - 1)
        return self.tiers[tier].draft_tokens

    def batch_schedule(self) -> list[list[int]]:
        """Rows ``[first_batch, last_batch, draft_tokens]`` (inclusive bounds)."""
        firsts = [1] + [t.max_batch + 1 for t in self.tiers[:-1]]
        return [[lo, t.max_batch, t.draft_tokens] for lo, t in zip(firsts, self.tiers)]


@dataclass(frozen=True, slots=True)
class DraftModelSpeculationConfig:
    draft_tokens: int = 4
    single_request_only: bool = True
    confidence_threshold: float | None = None

    def __post_init__(self) -> None:
        if self.draft_tokens < 1:
            raise ValueError("draft_tokens has to be positive")
        if self.confidence_threshold is not None and not 0.0 < self.confidence_threshold < 1.0:
            raise ValueError("confidence_threshold lies strictly between 0 and 1")


@dataclass(frozen=True, slots=True)
class DraftProposal:
    token_ids: TokenSequence
    token_probabilities: tuple[float, ...]
    matched_context_tokens: int
    token_distributions: tuple[tuple[tuple[int, float], ...], ...] = ()

    @property
    def stochastic(self) -> bool:
        return bool(self.token_distributions)


@dataclass(frozen=True, slots=True)
class RolloutTokenTreeSnapshot:
    observed_sequences: int
    observed_tokens: int
    contexts: int
    evicted_contexts: int
    queries: int
    hits: int
    proposed_tokens: int
    accepted_tokens: int
    rejected_tokens: int

    @property
    def hit_rate(self) -> float:
        return self.hits / self.queries if self.queries else 0.0

    @property
    def acceptance_rate(self) -> float:
        judged = self.accepted_tokens + self.rejected_tokens
        return self.accepted_tokens / judged if judged else 0.0


class RolloutTokenTree:
    """Contexts of ``min_context_tokens .. max_context_tokens`` tokens mapped to next-token
    counts, bounded by ``max_contexts`` with least-recently-used eviction.  A draft step
    uses the longest context that matches the end of the current text."""

    def __init__(self, *, max_context_tokens: int = 24, max_contexts: int = 100_000, min_context_tokens: int = 2,
                 min_token_probability: float = 0.1):
        if max_context_tokens < 1 or max_contexts < 1:
            raise ValueError("context length and context budget must be positive")
        if not 1 <= min_context_tokens <= max_context_tokens:
            raise ValueError("min_context_tokens must lie in 1..max_context_tokens")
        if not 0.0 <= min_token_probability <= 1.0:
            raise ValueError("min_token_probability is a probability")
        self.max_context_tokens = int(max_context_tokens)
        self.max_contexts = int(max_contexts)
        self.min_context_tokens = int(min_context_tokens)
        self.min_token_probability = float(min_token_probability)
        self._table: OrderedDict[tuple, Counter] = OrderedDict()
        self._lock = threading.RLock()
        self._stats = Counter()

    @classmethod
    def from_config(cls, config: ActiveBatchSpeculationConfig) -> "RolloutTokenTree":
        return cls(max_context_tokens=config.tree_max_context_tokens, max_contexts=config.tree_max_contexts,
                   min_context_tokens=config.min_context_tokens, min_token_probability=config.min_token_probability)

    def _touch(self, context: tuple) -> Counter:
        counts = self._table.get(context)
        if counts is None:
            counts = self._table[context] = Counter()
        else:
            self._table.move_to_end(context)
        return counts

    def observe(self, tokens: TokenSequence) -> None:
        seq = tuple(int(t) for t in tokens)
        lo, hi = self.min_context_tokens, self.max_context_tokens
        if len(seq) <= lo:
            return
        with self._lock:
            self._stats["sequences"] += 1
            self._stats["tokens"] += len(seq)
            for end in range(lo, len(seq)):
                following = seq[end]
                for width in range(lo, min(hi, end) + 1):
                    self._touch(seq[end - width:end])[following] += 1
            excess = len(self._table) - self.max_contexts
            for _ in range(max(0, excess)):
                self._table.popitem(last=False)
            self._stats["evicted"] += max(0, excess)

    def observe_sample(self, sample: SequenceSample) -> None:
        self.observe(sample.full_sequence)

    def observe_samples(self, samples: Iterable[SequenceSample]) -> None:
        for sample in samples:
            self.observe_sample(sample)

    def _longest_match(self, text: list[int]) -> tuple[Counter | None, int]:
        for width in range(min(self.max_context_tokens, len(text)), self.min_context_tokens - 1, -1):
            context = tuple(text[-width:])
            counts = self._table.get(context)
            if counts:
                self._table.move_to_end(context)
                return counts, width
        return None, 0

    def draft(self, prefix: TokenSequence, max_tokens: int, *, stochastic: bool = False, seed: int | None = None
              ) -> DraftProposal:
        """Extend ``prefix`` by the most frequent (or, with ``stochastic``, a sampled) next token
        of the longest matching context, for up to ``max_tokens`` tokens."""
        if max_tokens < 0:
            raise ValueError("max_tokens cannot be negative")
        if stochastic and seed is None:
            raise ValueError("a stochastic draft needs an explicit seed")
        if seed is not None and seed < 0:
            raise ValueError("the draft seed cannot be negative")
        if max_tokens == 0:
            return DraftProposal((), (), 0)
        rng = np.random.default_rng(seed) if stochastic else None
        text = [int(t) for t in prefix]
        drafted: list[int] = []
        probabilities: list[float] = []
        laws: list[tuple] = []
        first_width = 0
        with self._lock:
            self._stats["queries"] += 1
            while len(drafted) < max_tokens:
                counts, width = self._longest_match(text)
                if counts is None:
                    break
                tokens = np.asarray(sorted(counts), dtype=np.int64)
                mass = np.asarray([counts[t] for t in tokens], dtype=np.float64)
                mass /= mass.sum()
                if mass.max() < self.min_token_probability:
                    break
                if rng is not None:
                    pick = int(rng.choice(tokens.size, p=mass))
                    laws.append(tuple(zip(tokens.tolist(), mass.tolist())))
                else:
                    pick = int(np.argmax(mass))      # first maximum: the smallest token id among ties
                if not drafted:
                    first_width = width
                drafted.append(int(tokens[pick]))
                probabilities.append(float(mass[pick]))
                text.append(int(tokens[pick]))
            if drafted:
                self._stats["hits"] += 1
                self._stats["proposed"] += len(drafted)
        return DraftProposal(tuple(drafted), tuple(probabilities), first_width, tuple(laws))

    def record_verification(self, *, proposed: int, accepted: int) -> None:
        if not 0 <= accepted <= proposed:
            raise ValueError("accepted drafts are a part of the proposed ones")
        with self._lock:
            self._stats["accepted"] += accepted
            self._stats["rejected"] += proposed - accepted

    def snapshot(self) -> RolloutTokenTreeSnapshot:
        with self._lock:
            s = self._stats
            return RolloutTokenTreeSnapshot(s["sequences"], s["tokens"], len(self._table), s["evicted"], s["queries"],
                                            s["hits"], s["proposed"], s["accepted"], s["rejected"])


def sample_batch_with_callback(backend: AutoregressiveBackend, requests: Sequence[GenerationRequest],
                               on_complete: SampleCompletionCallback) -> list[SequenceSample]:
    """Use the backend's streaming hook when it has one; otherwise report in batch order."""
    streaming = getattr(backend, "sample_batch_with_callback", None)
    if callable(streaming):
        return list(streaming(requests, on_complete))
    samples = backend.sample_batch(requests)
    for index, sample in enumerate(samples):
        on_complete(index, sample)
    return samples


@dataclass(frozen=True, slots=True)
class StreamingRewardSnapshot:
    generation_seconds: float
    reward_tail_seconds: float
    submitted_rewards: int


class StreamingRewardEvaluator:
    """Overlaps reward computation with generation on a thread pool."""

    def __init__(self, *, workers: int = 4):
        if workers < 1:
            raise ValueError("the reward pool needs at least one worker")
        self._pool = ThreadPoolExecutor(max_workers=int(workers), thread_name_prefix="osb-reward")
        self._closed = False

    def sample_and_score(self, backend, requests: Sequence[GenerationRequest],
                         reward_inputs: Sequence[tuple[TokenSequence, TokenSequence]], reward: TokenReward,
                         on_generation_complete: Callable[[Sequence[SequenceSample]], None] | None = None):
        if self._closed:
            raise RuntimeError("the streaming reward evaluator was closed")
        if len(requests) != len(reward_inputs):
            raise ValueError(f"{len(reward_inputs)} reward inputs for {len(requests)} requests")
        pending: dict[int, Future] = {}
        guard = threading.Lock()

        def finished(index: int, sample: SequenceSample) -> None:
            prompt, generated = reward_inputs[index]
            with guard:
                if index in pending:
                    raise RuntimeError(f"request {index} was reported finished twice")
                pending[index] = self._pool.submit(reward, prompt, tuple(generated) + tuple(sample.token_ids))

        started = time.perf_counter()
        samples = sample_batch_with_callback(backend, requests, finished)
        generated_at = time.perf_counter()
        if on_generation_complete is not None:
            on_generation_complete(samples)
        if len(samples) != len(requests) or len(pending) != len(requests):
            raise RuntimeError("the backend did not finish every request of the batch")
        rewards = tuple(float(pending[i].result()) for i in range(len(requests)))
        if not all(isfinite(r) for r in rewards):
            raise ValueError("a reward is not finite")
        return samples, rewards, StreamingRewardSnapshot(generated_at - started, time.perf_counter() - generated_at,
                                                         len(rewards))

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            self._pool.shutdown(wait=True)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


@dataclass(frozen=True, slots=True)
class RunAheadSnapshot:
    submitted_requests: int
    completed_requests: int
    completed_tokens: int
    failed_requests: int
    queued_requests: int
    critical_calls: int
    critical_wait_seconds: float


class _Turnstile:
    """Foreground calls have priority: background work starts only while no foreground
    call is active or waiting, and a foreground call waits only for the background
    chunk already running."""

    def __init__(self):
        self._cv = threading.Condition()
        self.foreground = 0          # active or waiting foreground calls
        self.background = False
        self.closed = False
        self.waited = 0.0
        self.calls = 0

    def foreground_enter(self) -> None:
        t0 = time.perf_counter()
        with self._cv:
            self.foreground += 1
            while self.background:
                self._cv.wait()
            self.calls += 1
            self.waited += time.perf_counter() - t0

    def foreground_leave(self) -> None:
        with self._cv:
            self.foreground -= 1
            self._cv.notify_all()

    def background_enter(self) -> bool:
        with self._cv:
            while not self.closed and self.foreground:
                self._cv.wait()
            if self.closed:
                return False
            self.background = True
            return True

    def background_leave(self) -> None:
        with self._cv:
            self.background = False
            self._cv.notify_all()

    def close(self) -> bool:
        with self._cv:
            was_open = not self.closed
            self.closed = True
            self._cv.notify_all()
            return was_open


class LowPriorityRunAheadBackend:
    """Background run-ahead generation that only feeds the draft tree; foreground calls preempt it."""

    def __init__(self, backend: AutoregressiveBackend, tree: RolloutTokenTree | None, *, chunk_tokens: int = 32,
                 queue_limit: int = 1024, outputs_already_observed: bool = False):
        if chunk_tokens < 1 or queue_limit < 1:
            raise ValueError("chunk_tokens and queue_limit must be positive")
        if tree is None and not outputs_already_observed:
            raise ValueError("run-ahead output goes to a token tree, unless the backend records it itself")
        self.backend = backend
        self.tree = tree
        self.chunk_tokens = int(chunk_tokens)
        self._self_observing = bool(outputs_already_observed)
        self._work: queue.Queue = queue.Queue(queue_limit)
        self._gate = _Turnstile()
        self._counts = Counter()
        self._counts_lock = threading.Lock()
        self._worker = threading.Thread(target=self._loop, name="osb-runahead", daemon=True)
        self._worker.start()

    @property
    def model_id(self) -> str:
        return self.backend.model_id

    def __getattr__(self, name: str) -> Any:
        return getattr(self.backend, name)

    def _count(self, key: str, n: int = 1) -> None:
        with self._counts_lock:
            self._counts[key] += n

    def submit_run_ahead(self, requests: Sequence[GenerationRequest]) -> int:
        if self._gate.closed:
            raise RuntimeError("the run-ahead backend was closed")
        accepted = 0
        for request in requests:
            try:
                self._work.put_nowait(request)
            except queue.Full:
                break
            accepted += 1
        self._count("submitted", accepted)
        return accepted

    def _foreground(self, call, *args):
        self._gate.foreground_enter()
        try:
            return call(*args)
        finally:
            self._gate.foreground_leave()

    def sample_batch(self, requests):
        return self._foreground(self.backend.sample_batch, requests)

    def sample_batch_with_callback(self, requests, on_complete):
        return self._foreground(sample_batch_with_callback, self.backend, requests, on_complete)

    def score_batch(self, requests):
        return self._foreground(self.backend.score_batch, requests)

    @staticmethod
    def _continuation_seed(seed: int, generated: int) -> int:
        state = np.random.SeedSequence([int(seed), int(generated)]).generate_state(1, dtype=np.uint64)[0]
        return int(state % np.uint64(2 ** 63 - 1))

    def _one_chunk(self, request: GenerationRequest) -> None:
        size = min(self.chunk_tokens, request.max_new_tokens)
        uniforms = None if request.uniforms is None else request.uniforms[:size]
        sample = self.backend.sample_batch([GenerationRequest(request.prefix, size, request.sampling, request.seed,
                                                              request.request_id, uniforms)])[0]
        if not self._self_observing:
            self.tree.observe_sample(sample)
        self._count("tokens", len(sample.token_ids))
        left = request.max_new_tokens - len(sample.token_ids)
        eos = request.sampling.eos_token_id
        if left <= 0 or (eos is not None and eos in sample.token_ids):
            self._count("completed")
            return
        rest = GenerationRequest(request.prefix + tuple(sample.token_ids), left, request.sampling,
                                 self._continuation_seed(request.seed, len(sample.token_ids)), request.request_id,
                                 None if request.uniforms is None else request.uniforms[size:])
        try:                                    # the remainder is a later, preemptible chunk
            self._work.put_nowait(rest)
        except queue.Full:
            pass

    def _loop(self) -> None:
        while True:
            request = self._work.get()
            if request is None or not self._gate.background_enter():
                return
            try:
                self._one_chunk(request)
            except Exception:   # noqa: BLE001 - a failed background chunk must not stop the worker
                self._count("failed")
            finally:
                self._gate.background_leave()

    def wait_for_run_ahead(self, timeout: float = 60.0) -> None:
        deadline = time.monotonic() + timeout
        while time.monotonic() < deadline and (not self._work.empty() or self._gate.background):
            time.sleep(0.005)

    def snapshot(self) -> RunAheadSnapshot:
        with self._counts_lock:
            c = Counter(self._counts)
        return RunAheadSnapshot(c["submitted"], c["completed"], c["tokens"], c["failed"], self._work.qsize(),
                                self._gate.calls, self._gate.waited)

    def close(self) -> None:
        if not self._gate.close():
            return
        try:
            self._work.put_nowait(None)
        except queue.Full:
            pass
        self._worker.join(timeout=30)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()


__all__ = ["ActiveBatchSpeculationConfig", "DraftModelSpeculationConfig", "DraftProposal", "LowPriorityRunAheadBackend",
           "RolloutTokenTree", "RolloutTokenTreeSnapshot", "RunAheadSnapshot", "SpeculationTier",
           "StreamingRewardEvaluator", "StreamingRewardSnapshot", "sample_batch_with_callback"]
