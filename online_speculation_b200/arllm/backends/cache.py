"""Least-recently-used cache of exact continuation scores.

Scores are deterministic functions of (sampling policy, prefix, continuation), so a
repeated triple is answered from memory and only the misses reach the wrapped backend,
one request per distinct (policy, prefix).  Generations are random and never cached.
Interface of src/inference_scaling/arllm/backends/cache.py (ScoreCachingBackend and
its snapshot fields).
"""

from __future__ import annotations

import threading
from collections import OrderedDict
from collections.abc import Sequence
from dataclasses import dataclass

from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample


@dataclass(frozen=True, slots=True)
class ScoreCacheSnapshot:
    entries: int
    hits: int
    misses: int
    evictions: int

    @property
    def hit_rate(self) -> float:
        looked_up = self.hits + self.misses
        return self.hits / looked_up if looked_up else 0.0


class _LRU:
    def __init__(self, capacity: int):
        self.capacity = capacity
        self.items: OrderedDict = OrderedDict()
        self.evictions = 0

    def get(self, key):
        value = self.items.get(key)
        if value is not None:
            self.items.move_to_end(key)
        return value

    def put_if_absent(self, key, value):
        """Store ``value`` unless another thread stored one first; returns the stored value."""
        held = self.get(key)
        if held is not None:
            return held
        self.items[key] = value
        while len(self.items) > self.capacity:
            self.items.popitem(last=False)
            self.evictions += 1
        return value


class ScoreCachingBackend:
    def __init__(self, backend: AutoregressiveBackend, *, maximum_entries: int = 100_000):
        if maximum_entries < 1:
            raise ValueError("the score cache needs room for at least one entry")
        self._backend = backend
        self._lru = _LRU(int(maximum_entries))
        self._lock = threading.RLock()
        self._hits = 0
        self._misses = 0

    @property
    def model_id(self) -> str:
        return self._backend.model_id

    @property
    def backend(self):
        return self._backend

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        return self._backend.sample_batch(requests)

    def _score_misses(self, misses: dict) -> dict:
        by_context: dict[tuple, list] = {}
        for policy, prefix, continuation in misses:
            by_context.setdefault((policy, prefix), []).append(continuation)
        batch = [ScoreRequest(prefix, tuple(conts), policy) for (policy, prefix), conts in by_context.items()]
        keys = [(policy, prefix, c) for (policy, prefix), conts in by_context.items() for c in conts]
        scores = self._backend.score_batch(batch)
        if len(scores) != len(keys):
            raise RuntimeError(f"the wrapped backend returned {len(scores)} scores for {len(keys)} continuations")
        fresh = {}
        with self._lock:
            for key, value in zip(keys, scores):
                if len(value) != len(key[2]):
                    raise RuntimeError("a score does not have one entry per continuation token")
                fresh[key] = self._lru.put_if_absent(key, value)
        return fresh

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        wanted = [(r.sampling, r.prefix, c) for r in requests for c in r.continuations]
        known: dict = {}
        misses: dict = {}
        with self._lock:
            for key in wanted:
                value = self._lru.get(key)
                if value is None:
                    self._misses += 1
                    misses[key] = None
                else:
                    self._hits += 1
                    known[key] = value
        if misses:
            known.update(self._score_misses(misses))
        return [known[key] for key in wanted]

    def clear(self) -> None:
        with self._lock:
            self._lru.items.clear()

    def snapshot(self) -> ScoreCacheSnapshot:
        with self._lock:
            return ScoreCacheSnapshot(len(self._lru.items), self._hits, self._misses, self._lru.evictions)


__all__ = ["ScoreCacheSnapshot", "ScoreCachingBackend"]
