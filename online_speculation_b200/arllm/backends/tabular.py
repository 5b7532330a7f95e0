"""Exact finite autoregressive backends for distributional tests (CPU oracle).

``TabularBackend`` evaluates an arbitrary next-token law ``row(prefix)`` and
applies the real policy transforms (temperature, top-k, top-p), so algorithms
see genuine behaviour-policy probabilities and targets can be enumerated.
Two constructors cover the reference's prefix-keyed table
(src/inference_scaling/arllm/backends/tabular.py:30-195) and the
position-indexed toy model whose logits do not depend on the prefix:
``per_position_logits(vocab, length, seed)`` draws N(0, 1) logits per position.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence

import numpy as np

from ...shared.types import TokenSequence
from ..config import SamplingConfig
from ..types import GenerationRequest, ScoreRequest, SequenceSample


def _normalize(p: np.ndarray) -> np.ndarray:
    total = float(p.sum())
    if not np.isfinite(total) or total <= 0:
        raise ValueError("probabilities must have a positive finite sum")
    return p / total


def apply_policy(base: np.ndarray, sampling: SamplingConfig | None) -> np.ndarray:
    """Temperature, top-k and nucleus truncation of a probability vector."""
    if sampling is None:
        return base.copy()
    out = np.zeros_like(base)
    pos = base > 0
    out[pos] = np.exp(np.log(base[pos]) / sampling.temperature)
    V = base.shape[0]
    if sampling.top_k is not None and sampling.top_k < V:
        keep = np.argpartition(out, -sampling.top_k)[-sampling.top_k:]
        mask = np.zeros(V, dtype=bool)
        mask[keep] = True
        out[~mask] = 0
    out = _normalize(out)
    if sampling.top_p < 1:
        order = np.argsort(-out, kind="stable")
        count = int(np.searchsorted(np.cumsum(out[order]), sampling.top_p, side="left")) + 1
        mask = np.zeros(V, dtype=bool)
        mask[order[:count]] = True
        out[~mask] = 0
        out = _normalize(out)
    return out


class TabularBackend:
    """Exact sampler/scorer over a finite vocabulary given ``row(prefix) -> probs``."""

    def __init__(self, row: Callable[[TokenSequence], np.ndarray], vocab_size: int, *, model_id: str = "tabular",
                 prompt_length: int = 0):
        self._row = row
        self.vocab_size = int(vocab_size)
        self._model_id = model_id
        self.prompt_length = prompt_length
        self.sampled_tokens = 0

    @classmethod
    def from_table(cls, table: Mapping[TokenSequence, Sequence[float]], *, fallback: Sequence[float] | None = None,
                   model_id: str = "tabular") -> "TabularBackend":
        rows = {tuple(k): _normalize(np.asarray(v, dtype=np.float64)) for k, v in table.items()}
        fb = None if fallback is None else _normalize(np.asarray(fallback, dtype=np.float64))
        first = next(iter(rows.values()), fb)
        if first is None:
            raise ValueError("at least one transition or a fallback distribution is required")
        for r in rows.values():
            if r.shape != first.shape or np.any(r < 0):
                raise ValueError("all transition rows must share one non-negative vocabulary")

        def row(prefix):
            if prefix in rows:
                return rows[prefix]
            if fb is not None:
                return fb
            raise KeyError(f"no transition probabilities for prefix {prefix!r}")

        return cls(row, first.shape[0], model_id=model_id)

    @classmethod
    def per_position_logits(cls, vocab: int, length: int, seed: int, *, prompt_length: int = 0,
                            model_id: str = "tabular-positional") -> "TabularBackend":
        """Position-indexed model: logits[t] ~ N(0, 1) i.i.d., independent of the prefix."""
        logits = np.random.default_rng(seed).standard_normal((length, vocab))
        probs = np.exp(logits - logits.max(-1, keepdims=True))
        probs /= probs.sum(-1, keepdims=True)
        backend = cls(lambda prefix: probs[min(len(prefix) - prompt_length, length - 1)], vocab,
                      model_id=model_id, prompt_length=prompt_length)
        backend.position_probabilities = probs
        return backend

    @property
    def model_id(self) -> str:
        return self._model_id

    def probabilities(self, prefix: TokenSequence, sampling: SamplingConfig | None = None) -> np.ndarray:
        return apply_policy(self._row(tuple(prefix)), sampling)

    def next_token_probabilities(self, prefix: TokenSequence, block: TokenSequence = ()) -> np.ndarray:
        """Temperature-1 distributions after prefix + block[:i] for i = 0..len(block), [len(block) + 1, V]."""
        ctx = tuple(prefix)
        block = tuple(block)
        return np.stack([self._row(ctx + block[:i]) for i in range(len(block) + 1)]).astype(np.float64)

    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        out = []
        for req in requests:
            rng = np.random.default_rng(req.seed)
            arith = req.arithmetic_uniform
            ctx = list(req.prefix)
            toks, logq, logp = [], [], []
            finish = "length"
            for step in range(req.max_new_tokens):
                base = self._row(tuple(ctx))
                probs = apply_policy(base, req.sampling)
                if arith is not None:
                    order = np.argsort(-probs, kind="stable")
                    cdf = np.cumsum(probs[order])
                    cdf[-1] = 1.0
                    rank = min(int(np.searchsorted(cdf, arith, side="right")), self.vocab_size - 1)
                    tok = int(order[rank])
                    lower = 0.0 if rank == 0 else float(cdf[rank - 1])
                    arith = min(max((arith - lower) / float(probs[tok]), 0.0), float(np.nextafter(1.0, 0.0)))
                elif req.uniforms is None:
                    tok = int(rng.choice(self.vocab_size, p=probs))
                else:
                    tok = min(int(np.searchsorted(np.cumsum(probs), req.uniforms[step], side="right")),
                              self.vocab_size - 1)
                toks.append(tok)
                logq.append(float(np.log(probs[tok])))
                logp.append(float(np.log(base[tok])) if base[tok] > 0 else float("-inf"))
                ctx.append(tok)
                if req.sampling.eos_token_id == tok:
                    finish = "eos"
                    break
            self.sampled_tokens += len(toks)
            finite_ref = all(np.isfinite(v) for v in logp)
            out.append(SequenceSample(req.prefix, tuple(toks), tuple(logq), req.sampling.policy_id, self.model_id,
                                      req.request_id, finish, tuple(logp) if finite_ref else None,
                                      SamplingConfig().policy_id if finite_ref else None))
        return out

    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        out = []
        for req in requests:
            for cont in req.continuations:
                ctx = list(req.prefix)
                vals = []
                for tok in cont:
                    p = float(self.probabilities(tuple(ctx), req.sampling)[tok])
                    vals.append(float("-inf") if p == 0 else float(np.log(p)))
                    ctx.append(tok)
                out.append(tuple(vals))
        return out


def _tabular_statistics(self, requests, *, confidence_top_k=None):
    """Exact per-token statistics (entropy, self-certainty, top-K confidence) of the tabular model."""
    from ...engine.backend import SequenceScoreStatistics

    out = []
    for req in requests:
        pol = req.sampling or SamplingConfig()
        if not pol.full_support:
            raise ValueError("entropy and self-certainty require a full-support policy")
        for cont in req.continuations:
            if not cont:
                raise ValueError("confidence rewards require nonempty continuations")
            ctx = list(req.prefix)
            lps, negent, cert, conf = [], [], [], []
            for tok in cont:
                p = self.probabilities(tuple(ctx), pol)
                lp = np.log(np.maximum(p, 1e-300))
                lps.append(float(lp[tok]))
                negent.append(float((p * lp).sum()))
                cert.append(float(-(np.log(self.vocab_size) + lp.mean())))
                if confidence_top_k:
                    k = min(confidence_top_k, self.vocab_size)
                    conf.append(float(-np.sort(lp)[-k:].mean()))
                ctx.append(tok)
            n = len(cont)
            out.append(SequenceScoreStatistics(tuple(lps), sum(lps) / n, sum(negent) / n, sum(cert) / n, tuple(conf),
                                               confidence_top_k))
    return out


TabularBackend.score_statistics_batch = _tabular_statistics
