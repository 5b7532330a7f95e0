"""Cross-caller continuous batching for synchronous algorithm code.

Independent prompt workers (threads) call ``sample_batch`` / ``score_batch`` as
usual; a background thread merges caller groups that arrive within
``batch_wait_seconds`` and share a batch key (same sampling policy, same
generation length, same repeated-prefix structure for sampling; same policy
and a 64-token length bucket for scoring) into one backend call, within
``max_batch_size`` sequences and ``max_batch_tokens``.  Caller groups stay
intact (so shared prefixes keep their KV reuse); an oversized group is split
at repeated-prefix run boundaries where possible.  Random streams are
request-local, so merging does not change any sample.  A backend that
batches natively (``supports_native_continuous_batching``) is passed through.

Reference behaviour: src/inference_scaling/arllm/backends/batching.py:53-480.
"""

from __future__ import annotations

import queue
import threading
import time
from collections import Counter
from collections.abc import Sequence
from concurrent.futures import Future
from dataclasses import dataclass

from ..types import AutoregressiveBackend, GenerationRequest, ScoreRequest, SequenceSample

_STOP = object()


@dataclass(slots=True)
class _Group:
    kind: str
    requests: tuple
    future: Future
    sequences: int
    tokens: int
    key: tuple


@dataclass(frozen=True, slots=True)
class BatchingSnapshot:
    sample_batches: int
    score_batches: int
    sample_requests: int
    score_sequences: int
    maximum_sample_batch: int
    maximum_score_batch: int

    @property
    def average_sample_batch(self) -> float:
        return self.sample_requests / self.sample_batches if self.sample_batches else 0.0

    @property
    def average_score_batch(self) -> float:
        return self.score_sequences / self.score_batches if self.score_batches else 0.0


def _gen_cost(r: GenerationRequest) -> int:
    return max(1, len(r.prefix) + r.max_new_tokens)


def _score_cost(r: ScoreRequest) -> int:
    return max(1, sum(len(r.prefix) + len(c) for c in r.continuations))


class ContinuousBatchingBackend:
    def __init__(self, backend: AutoregressiveBackend, *, max_batch_size: int = 32, max_batch_tokens: int = 4096,
                 batch_wait_seconds: float = 0.002):
        if max_batch_size <= 0 or max_batch_tokens <= 0:
            raise ValueError("batch limits must be positive")
        if batch_wait_seconds < 0:
            raise ValueError("batch_wait_seconds must be non-negative")
        self._backend = backend
        self._native = bool(getattr(backend, "supports_native_continuous_batching", False))
        self._max_seq, self._max_tok, self._wait = int(max_batch_size), int(max_batch_tokens), float(batch_wait_seconds)
        self._q: queue.Queue = queue.Queue()
        self._lock = threading.Lock()
        self._stats_lock = threading.Lock()
        self._closed = False
        self._stats = Counter()
        self._worker = None
        if not self._native:
            self._worker = threading.Thread(target=self._run, name=f"batching:{backend.model_id}", daemon=True)
            self._worker.start()

    @property
    def model_id(self) -> str:
        return self._backend.model_id

    @property
    def backend(self):
        return self._backend

    def _fits(self, seqs: int, toks: int) -> bool:
        return seqs <= self._max_seq and toks <= self._max_tok

    # ---- caller side ----
    def _submit(self, g: _Group) -> Future:
        with self._lock:
            if self._closed:
                raise RuntimeError("continuous batching backend is closed")
            self._q.put(g)
        return g.future

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        if not requests:
            return []
        if self._native:
            self._check_open()
            self._record("sample", len(requests))
            return self._backend.sample_batch(requests)
        futs = [self._submit(_Group("sample", g, Future(), len(g), sum(_gen_cost(r) for r in g), self._sample_key(g)))
                for g in self._split_sample(tuple(requests))]
        return [s for f in futs for s in f.result()]

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        if not requests:
            return []
        if self._native:
            self._check_open()
            self._record("score", sum(len(r.continuations) for r in requests))
            return self._backend.score_batch(requests)
        futs = [self._submit(_Group("score", g, Future(), sum(len(r.continuations) for r in g),
                                    sum(_score_cost(r) for r in g), self._score_key(g)))
                for g in self._split_score(tuple(requests))]
        return [v for f in futs for v in f.result()]

    def _check_open(self):
        with self._lock:
            if self._closed:
                raise RuntimeError("continuous batching backend is closed")

    @staticmethod
    def _sample_key(g) -> tuple:
        s0, n0 = g[0].sampling, g[0].max_new_tokens
        reps = set(Counter(r.prefix for r in g).values())
        return ("sample", s0 if all(r.sampling == s0 for r in g) else None,
                n0 if all(r.max_new_tokens == n0 for r in g) else None, reps.pop() if len(reps) == 1 else None)

    @staticmethod
    def _score_key(g) -> tuple:
        s0 = g[0].sampling
        longest = max((len(r.prefix) + len(c) for r in g for c in r.continuations), default=0)
        return "score", s0 if all(r.sampling == s0 for r in g) else None, -(-longest // 64) * 64

    def _split_sample(self, reqs: tuple) -> list[tuple]:
        if self._fits(len(reqs), sum(_gen_cost(r) for r in reqs)):
            return [reqs]
        runs: list[list] = []
        last = None
        for r in reqs:                         # runs of identical (policy, prefix, length): keep together if possible
            k = (r.sampling, r.prefix, r.max_new_tokens)
            if k != last:
                runs.append([])
                last = k
            runs[-1].append(r)
        out, cur, cost = [], [], 0
        for run in runs:
            rest = list(run)
            while rest:
                rc = sum(_gen_cost(r) for r in rest)
                if self._fits(len(cur) + len(rest), cost + rc):
                    cur += rest
                    cost += rc
                    rest = []
                elif cur:
                    out.append(tuple(cur))
                    cur, cost = [], 0
                else:
                    take, tc = 0, 0
                    for r in rest:
                        c = _gen_cost(r)
                        if take and not self._fits(take + 1, tc + c):
                            break
                        take, tc = take + 1, tc + c
                    take = max(1, take)
                    out.append(tuple(rest[:take]))
                    rest = rest[take:]
        if cur:
            out.append(tuple(cur))
        return out

    def _split_score(self, reqs: tuple) -> list[tuple]:
        out, cur, seqs, toks = [], [], 0, 0
        for r in reqs:
            n, c = len(r.continuations), _score_cost(r)
            if cur and not self._fits(seqs + n, toks + c):
                out.append(tuple(cur))
                cur, seqs, toks = [], 0, 0
            cur.append(r)
            seqs, toks = seqs + n, toks + c
        if cur:
            out.append(tuple(cur))
        return out

    # ---- worker side ----
    def _record(self, kind: str, n: int) -> None:
        with self._stats_lock:
            self._stats[f"{kind}_batches"] += 1
            self._stats[f"{kind}_items"] += n
            self._stats[f"{kind}_max"] = max(self._stats[f"{kind}_max"], n)

    def _dispatch(self, batch: list[_Group]) -> None:
        kind = batch[0].kind
        total = sum(g.sequences for g in batch)
        self._record(kind, total)
        try:
            flat = [r for g in batch for r in g.requests]
            res = self._backend.sample_batch(flat) if kind == "sample" else self._backend.score_batch(flat)
            if len(res) != total:
                raise RuntimeError(f"underlying backend returned an invalid {kind} batch")
            off = 0
            for g in batch:
                g.future.set_result(list(res[off:off + g.sequences]))
                off += g.sequences
        except BaseException as e:   # noqa: BLE001 - every waiting caller must be released
            for g in batch:
                if not g.future.done():
                    g.future.set_exception(e)

    def _run(self) -> None:
        pending: list[_Group] = []
        stop = False
        while not stop or pending:
            if not pending:
                item = self._q.get()
                if item is _STOP:
                    stop = True
                    continue
                pending.append(item)
            deadline = time.monotonic() + self._wait
            while not stop:
                left = deadline - time.monotonic()
                try:
                    item = self._q.get(timeout=max(0.0, left)) if left > 0 else self._q.get_nowait()
                except queue.Empty:
                    break
                if item is _STOP:
                    stop = True
                    break
                pending.append(item)
            head = pending[0]
            batch, seqs, toks, rest = [head], head.sequences, head.tokens, []
            for g in pending[1:]:
                if g.kind == head.kind and g.key == head.key and self._fits(seqs + g.sequences, toks + g.tokens):
                    batch.append(g)
                    seqs, toks = seqs + g.sequences, toks + g.tokens
                else:
                    rest.append(g)
            pending = rest
            self._dispatch(batch)

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
        if self._worker is not None:
            self._q.put(_STOP)
            self._worker.join()

    def __del__(self):
        try:
            self.close()
        except Exception:   # noqa: BLE001 - interpreter shutdown
            pass

    def snapshot(self) -> BatchingSnapshot:
        s = self._stats
        return BatchingSnapshot(s["sample_batches"], s["score_batches"], s["sample_items"], s["score_items"],
                                s["sample_max"], s["score_max"])


__all__ = ["BatchingSnapshot", "ContinuousBatchingBackend"]
