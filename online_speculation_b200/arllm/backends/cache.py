"""Exact LRU cache of continuation scores keyed by (policy, prefix, continuation).

Generations are never cached (they are random); scores are deterministic, so a
repeated (policy, prefix, continuation) is served from the cache and only the
misses go to the wrapped backend, grouped by (policy, prefix).
Reference behaviour: src/inference_scaling/arllm/backends/cache.py:35-123.
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
        t = self.hits + self.misses
        return self.hits / t if t else 0.0


class ScoreCachingBackend:
    def __init__(self, backend: AutoregressiveBackend, *, maximum_entries: int = 100_000):
        if maximum_entries <= 0:
            raise ValueError("maximum_entries must be positive")
        self._backend, self._cap = backend, int(maximum_entries)
        self._cache: OrderedDict = OrderedDict()
        self._lock = threading.RLock()
        self._hits = self._misses = self._evictions = 0

    @property
    def model_id(self) -> str:
        return self._backend.model_id

    @property
    def backend(self):
        return self._backend

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        return self._backend.sample_batch(requests)

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        order, found, missing = [], {}, OrderedDict()
        with self._lock:
            for r in requests:
                for c in r.continuations:
                    key = (r.sampling, r.prefix, c)
                    order.append(key)
                    hit = self._cache.get(key)
                    if hit is None:
                        self._misses += 1
                        missing.setdefault(key, None)
                    else:
                        self._hits += 1
                        self._cache.move_to_end(key)
                        found[key] = hit
        if missing:
            groups: OrderedDict = OrderedDict()
            for s, p, c in missing:
                groups.setdefault((s, p), []).append(c)
            reqs = [ScoreRequest(p, tuple(cs), s) for (s, p), cs in groups.items()]
            keys = [(s, p, c) for (s, p), cs in groups.items() for c in cs]
            scored = self._backend.score_batch(reqs)
            if len(scored) != len(keys):
                raise RuntimeError("underlying backend returned an invalid score batch")
            with self._lock:
                for key, val in zip(keys, scored):
                    if len(val) != len(key[2]):
                        raise RuntimeError("underlying backend returned an invalid score shape")
                    old = self._cache.get(key)
                    if old is None:
                        self._cache[key] = val
                        while len(self._cache) > self._cap:
                            self._cache.popitem(last=False)
                            self._evictions += 1
                        found[key] = val
                    else:
                        self._cache.move_to_end(key)
                        found[key] = old
        return [found[k] for k in order]

    def clear(self) -> None:
        with self._lock:
            self._cache.clear()

    def snapshot(self) -> ScoreCacheSnapshot:
        with self._lock:
            return ScoreCacheSnapshot(len(self._cache), self._hits, self._misses, self._evictions)


__all__ = ["ScoreCacheSnapshot", "ScoreCachingBackend"]
