"""Rollout acceleration utilities that never change the sampled law.

* ``ActiveBatchSpeculationConfig``: draft length as a function of the active
  batch (speculate only in the long tail, where decoding is latency bound).
* ``RolloutTokenTree``: a bounded CPU suffix table of empirical next-token
  counts built from past rollouts; its drafts are always verified by the base
  model (``EngineBackend`` checks a draft token against the token its own
  inverse-CDF draw produces), so no draft probability ever enters an IS weight.
* ``StreamingRewardEvaluator``: CPU reward work starts as soon as each sequence
  finishes (thread pool), overlapping the rest of the GPU batch.
* ``LowPriorityRunAheadBackend``: fills the token tree in idle gaps with
  bounded, preemptible background chunks; foreground calls wait at most one
  chunk.

Reference behaviour: src/inference_scaling/arllm/acceleration.py:38-714.
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
    """At most ``draft_tokens`` drafts while the active batch is at most ``max_batch``."""

    max_batch: int
    draft_tokens: int

    def __post_init__(self) -> None:
        if self.max_batch <= 0:
            raise ValueError("max_batch must be positive")
        if self.draft_tokens < 0:
            raise ValueError("draft_tokens must be non-negative")


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
        if not self.tiers:
            raise ValueError("at least one speculation tier is required")
        if any(b.max_batch <= a.max_batch for a, b in zip(self.tiers, self.tiers[1:])):
            raise ValueError("speculation tiers must have increasing max_batch values")
        if self.min_context_tokens <= 0:
            raise ValueError("min_context_tokens must be positive")
        if not 0 <= self.min_token_probability <= 1:
            raise ValueError("min_token_probability must lie in [0, 1]")
        if self.tree_max_context_tokens <= 0 or self.tree_max_contexts <= 0:
            raise ValueError("token-tree limits must be positive")
        if self.vllm_max_cached_requests < 0:
            raise ValueError("vllm_max_cached_requests must be non-negative")

    @property
    def maximum_draft_tokens(self) -> int:
        return max(t.draft_tokens for t in self.tiers)

    def draft_tokens(self, active_batch: int) -> int:
        if active_batch <= 0:
            raise ValueError("active_batch must be positive")
        return next((t.draft_tokens for t in self.tiers if active_batch <= t.max_batch), self.tiers[-1].draft_tokens)

    def batch_schedule(self) -> list[list[int]]:
        """Inclusive ``[first_batch, last_batch, draft_tokens]`` rows."""
        rows, lo = [], 1
        for t in self.tiers:
            rows.append([lo, t.max_batch, t.draft_tokens])
            lo = t.max_batch + 1
        return rows


@dataclass(frozen=True, slots=True)
class DraftModelSpeculationConfig:
    draft_tokens: int = 4
    single_request_only: bool = True
    confidence_threshold: float | None = None

    def __post_init__(self) -> None:
        if self.draft_tokens <= 0:
            raise ValueError("draft_tokens must be positive")
        if self.confidence_threshold is not None and not 0 < self.confidence_threshold < 1:
            raise ValueError("confidence_threshold must lie strictly between zero and one")


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
        v = self.accepted_tokens + self.rejected_tokens
        return self.accepted_tokens / v if v else 0.0


class RolloutTokenTree:
    """LRU-bounded suffix contexts (lengths min..max) -> next-token counts."""

    def __init__(self, *, max_context_tokens: int = 24, max_contexts: int = 100_000, min_context_tokens: int = 2,
                 min_token_probability: float = 0.1):
        if max_context_tokens <= 0 or max_contexts <= 0:
            raise ValueError("token-tree limits must be positive")
        if not 0 < min_context_tokens <= max_context_tokens:
            raise ValueError("min_context_tokens must lie within the context limit")
        if not 0 <= min_token_probability <= 1:
            raise ValueError("min_token_probability must lie in [0, 1]")
        self.max_context_tokens, self.max_contexts = int(max_context_tokens), int(max_contexts)
        self.min_context_tokens, self.min_token_probability = int(min_context_tokens), float(min_token_probability)
        self._ctx: OrderedDict[TokenSequence, Counter] = OrderedDict()
        self._lock = threading.RLock()
        self._s = Counter()

    @classmethod
    def from_config(cls, config: ActiveBatchSpeculationConfig) -> "RolloutTokenTree":
        return cls(max_context_tokens=config.tree_max_context_tokens, max_contexts=config.tree_max_contexts,
                   min_context_tokens=config.min_context_tokens,
                   min_token_probability=config.min_token_probability)

    def observe(self, tokens: TokenSequence) -> None:
        vals = tuple(int(t) for t in tokens)
        if len(vals) <= self.min_context_tokens:
            return
        with self._lock:
            self._s["sequences"] += 1
            self._s["tokens"] += len(vals)
            for pos in range(self.min_context_tokens, len(vals)):
                nxt = vals[pos]
                for n in range(self.min_context_tokens, min(self.max_context_tokens, pos) + 1):
                    key = vals[pos - n:pos]
                    c = self._ctx.get(key)
                    if c is None:
                        c = self._ctx[key] = Counter()
                    else:
                        self._ctx.move_to_end(key)
                    c[nxt] += 1
            while len(self._ctx) > self.max_contexts:
                self._ctx.popitem(last=False)
                self._s["evicted"] += 1

    def observe_sample(self, sample: SequenceSample) -> None:
        self.observe(sample.full_sequence)

    def observe_samples(self, samples: Iterable[SequenceSample]) -> None:
        for s in samples:
            self.observe_sample(s)

    def draft(self, prefix: TokenSequence, max_tokens: int, *, stochastic: bool = False, seed: int | None = None
              ) -> DraftProposal:
        """Extend ``prefix`` by the most frequent (or a sampled) next token of the longest matching context."""
        if max_tokens < 0:
            raise ValueError("max_tokens must be non-negative")
        if max_tokens == 0:
            return DraftProposal((), (), 0)
        if stochastic and seed is None:
            raise ValueError("stochastic token-tree drafts require an explicit seed")
        if seed is not None and seed < 0:
            raise ValueError("draft seed must be non-negative")
        rng = np.random.default_rng(seed) if stochastic else None
        work = [int(t) for t in prefix]
        toks, probs, dists = [], [], []
        first_match = 0
        with self._lock:
            self._s["queries"] += 1
            for _ in range(max_tokens):
                counts, matched = None, 0
                for n in range(min(self.max_context_tokens, len(work)), self.min_context_tokens - 1, -1):
                    c = self._ctx.get(tuple(work[-n:]))
                    if c:
                        counts, matched = c, n
                        self._ctx.move_to_end(tuple(work[-n:]))
                        break
                if counts is None:
                    break
                total = sum(counts.values())
                dist = tuple((int(t), c / total) for t, c in sorted(counts.items()))
                if max(p for _, p in dist) < self.min_token_probability:
                    break
                if stochastic:
                    t = int(rng.choice([a for a, _ in dist], p=[b for _, b in dist]))
                    p = dict(dist)[t]
                    dists.append(dist)
                else:
                    t, c = min(counts.items(), key=lambda kv: (-kv[1], kv[0]))    # stable tie-break
                    p = c / total
                if not toks:
                    first_match = matched
                toks.append(t)
                probs.append(float(p))
                work.append(t)
            if toks:
                self._s["hits"] += 1
                self._s["proposed"] += len(toks)
        return DraftProposal(tuple(toks), tuple(probs), first_match, tuple(dists))

    def record_verification(self, *, proposed: int, accepted: int) -> None:
        if not 0 <= accepted <= proposed:
            raise ValueError("accepted drafts must lie within the proposal")
        with self._lock:
            self._s["accepted"] += accepted
            self._s["rejected"] += proposed - accepted

    def snapshot(self) -> RolloutTokenTreeSnapshot:
        with self._lock:
            s = self._s
            return RolloutTokenTreeSnapshot(s["sequences"], s["tokens"], len(self._ctx), s["evicted"], s["queries"],
                                            s["hits"], s["proposed"], s["accepted"], s["rejected"])


def sample_batch_with_callback(backend: AutoregressiveBackend, requests: Sequence[GenerationRequest],
                               on_complete: SampleCompletionCallback) -> list[SequenceSample]:
    """The backend's streaming hook when it has one, else an ordered batch."""
    cb = getattr(backend, "sample_batch_with_callback", None)
    if callable(cb):
        return list(cb(requests, on_complete))
    out = backend.sample_batch(requests)
    for i, s in enumerate(out):
        on_complete(i, s)
    return out


@dataclass(frozen=True, slots=True)
class StreamingRewardSnapshot:
    generation_seconds: float
    reward_tail_seconds: float
    submitted_rewards: int


class StreamingRewardEvaluator:
    def __init__(self, *, workers: int = 4):
        if workers <= 0:
            raise ValueError("workers must be positive")
        self._pool = ThreadPoolExecutor(max_workers=int(workers), thread_name_prefix="osb-reward")
        self._closed = False

    def sample_and_score(self, backend, requests: Sequence[GenerationRequest],
                         reward_inputs: Sequence[tuple[TokenSequence, TokenSequence]], reward: TokenReward,
                         on_generation_complete: Callable[[Sequence[SequenceSample]], None] | None = None):
        if self._closed:
            raise RuntimeError("streaming reward evaluator is closed")
        if len(requests) != len(reward_inputs):
            raise ValueError("reward_inputs must have one entry per request")
        futs: list[Future | None] = [None] * len(requests)
        lock = threading.Lock()

        def done(i, s):
            prompt, gen = reward_inputs[i]
            with lock:
                if futs[i] is not None:
                    raise RuntimeError("backend completed one request more than once")
                futs[i] = self._pool.submit(reward, prompt, gen + s.token_ids)

        t0 = time.perf_counter()
        samples = sample_batch_with_callback(backend, requests, done)
        t1 = time.perf_counter()
        if on_generation_complete is not None:
            on_generation_complete(samples)
        if len(samples) != len(requests) or any(f is None for f in futs):
            raise RuntimeError("backend returned an incomplete streaming batch")
        rewards = tuple(float(f.result()) for f in futs)
        if not all(isfinite(v) for v in rewards):
            raise ValueError("reward must be finite")
        return samples, rewards, StreamingRewardSnapshot(t1 - t0, time.perf_counter() - t1, len(rewards))

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


class LowPriorityRunAheadBackend:
    """Background run-ahead generation that only feeds the draft tree; foreground calls preempt it."""

    def __init__(self, backend: AutoregressiveBackend, tree: RolloutTokenTree | None, *, chunk_tokens: int = 32,
                 queue_limit: int = 1024, outputs_already_observed: bool = False):
        if chunk_tokens <= 0 or queue_limit <= 0:
            raise ValueError("run-ahead limits must be positive")
        if tree is None and not outputs_already_observed:
            raise ValueError("a draft tree is required unless the backend observes its own outputs")
        self.backend, self.tree = backend, tree
        self._observed = bool(outputs_already_observed)
        self.chunk_tokens = int(chunk_tokens)
        self._q: queue.Queue = queue.Queue(queue_limit)
        self._cv = threading.Condition()
        self._fg_wait = self._fg_active = 0
        self._bg_active = False
        self._closed = False
        self._c = Counter()
        self._wait_s = 0.0
        self._worker = threading.Thread(target=self._run, name="osb-runahead", daemon=True)
        self._worker.start()

    @property
    def model_id(self) -> str:
        return self.backend.model_id

    def __getattr__(self, name: str) -> Any:
        return getattr(self.backend, name)

    def submit_run_ahead(self, requests: Sequence[GenerationRequest]) -> int:
        with self._cv:
            if self._closed:
                raise RuntimeError("run-ahead backend is closed")
        n = 0
        for r in requests:
            try:
                self._q.put_nowait(r)
            except queue.Full:
                break
            n += 1
        with self._cv:
            self._c["submitted"] += n
            self._cv.notify_all()
        return n

    def _enter(self) -> None:
        t0 = time.perf_counter()
        with self._cv:
            self._fg_wait += 1
            try:
                while self._bg_active:
                    self._cv.wait()
                self._fg_active += 1
            finally:
                self._fg_wait -= 1
            self._c["critical"] += 1
            self._wait_s += time.perf_counter() - t0

    def _leave(self) -> None:
        with self._cv:
            self._fg_active -= 1
            self._cv.notify_all()

    def sample_batch(self, requests):
        self._enter()
        try:
            return self.backend.sample_batch(requests)
        finally:
            self._leave()

    def sample_batch_with_callback(self, requests, on_complete):
        self._enter()
        try:
            return sample_batch_with_callback(self.backend, requests, on_complete)
        finally:
            self._leave()

    def score_batch(self, requests):
        self._enter()
        try:
            return self.backend.score_batch(requests)
        finally:
            self._leave()

    @staticmethod
    def _continuation_seed(seed: int, generated: int) -> int:
        st = np.random.SeedSequence([int(seed), int(generated)]).generate_state(1, dtype=np.uint64)[0]
        return int(st % np.uint64(2 ** 63 - 1))

    def _run(self) -> None:
        while True:
            req = self._q.get()
            if req is None:
                return
            with self._cv:
                while not self._closed and (self._fg_active or self._fg_wait):
                    self._cv.wait()
                if self._closed:
                    return
                self._bg_active = True
            try:
                n = min(self.chunk_tokens, req.max_new_tokens)
                s = self.backend.sample_batch([GenerationRequest(
                    req.prefix, n, req.sampling, req.seed, req.request_id,
                    req.uniforms[:n] if req.uniforms is not None else None)])[0]
                if not self._observed:
                    self.tree.observe_sample(s)
                with self._cv:
                    self._c["tokens"] += len(s.token_ids)
                eos = req.sampling.eos_token_id
                left = req.max_new_tokens - len(s.token_ids)
                if left > 0 and not (eos is not None and eos in s.token_ids):
                    try:                                   # continue in a later, preemptible chunk
                        self._q.put_nowait(GenerationRequest(
                            req.prefix + s.token_ids, left, req.sampling,
                            self._continuation_seed(req.seed, len(s.token_ids)), req.request_id,
                            req.uniforms[n:] if req.uniforms is not None else None))
                    except queue.Full:
                        pass
                else:
                    with self._cv:
                        self._c["completed"] += 1
            except Exception:   # noqa: BLE001 - background work must not kill the worker
                with self._cv:
                    self._c["failed"] += 1
            finally:
                with self._cv:
                    self._bg_active = False
                    self._cv.notify_all()

    def wait_for_run_ahead(self, timeout: float = 60.0) -> None:
        end = time.monotonic() + timeout
        while time.monotonic() < end:
            with self._cv:
                if self._q.empty() and not self._bg_active:
                    return
            time.sleep(0.005)

    def snapshot(self) -> RunAheadSnapshot:
        with self._cv:
            c = self._c
            return RunAheadSnapshot(c["submitted"], c["completed"], c["tokens"], c["failed"], self._q.qsize(),
                                    c["critical"], self._wait_s)

    def close(self) -> None:
        with self._cv:
            if self._closed:
                return
            self._closed = True
            self._cv.notify_all()
        try:
            self._q.put_nowait(None)
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
