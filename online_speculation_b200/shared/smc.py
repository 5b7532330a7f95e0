"""Sequential Monte Carlo helpers: weight normalisation, systematic resampling,
and splitting replay reservoirs among resampled copies.

Systematic resampling is written in its counting form: with cumulative
probabilities C_i and one uniform u, branch i receives
``ceil(N C_i - u) - ceil(N C_{i-1} - u)`` of the N grid points (u + k) / N, so the
selected indices come out sorted from one ``np.repeat``.  The function names
follow src/inference_scaling/shared/smc.py (used by the SMC forest samplers).
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np


def normalize_smc_log_weights(log_weights: Sequence[float]) -> tuple[tuple[float, ...], float]:
    """Normalised probabilities and the effective sample size 1 / sum(p^2)."""
    v = np.asarray(list(log_weights), dtype=np.float64)
    if v.size == 0:
        raise ValueError("normalising SMC weights needs at least one branch")
    if not np.isfinite(v).all():
        raise ValueError("SMC log weights have to be finite")
    p = np.exp(v - v.max())
    p /= p.sum()
    if not np.isfinite(p).all():
        raise ValueError("SMC weights could not be normalised")
    return tuple(p.tolist()), float(1.0 / np.dot(p, p))


def systematic_resample(probabilities: Sequence[float], count: int, generator: np.random.Generator) -> tuple[int, ...]:
    """Indices of ``count`` systematic draws (one uniform from ``generator``), in increasing order."""
    if count < 1:
        raise ValueError("systematic resampling draws at least one index")
    p = np.asarray(list(probabilities), dtype=np.float64)
    if p.size == 0 or not np.isfinite(p).all() or (p < 0).any() or not p.sum() > 0:
        raise ValueError("resampling needs finite, non-negative probabilities with positive total mass")
    cdf = np.cumsum(p / p.sum())
    cdf[-1] = 1.0
    u = float(generator.random())
    # grid points strictly below N * C_i - u, i.e. (u + k) / N < C_i
    below = np.clip(np.ceil(count * cdf - u), 0, count).astype(np.int64)
    counts = np.diff(below, prepend=0)
    return tuple(np.repeat(np.arange(p.size), counts).tolist())


def partition_resampled_reservoirs(reservoirs: Sequence[Sequence], selected: Sequence[int]) -> tuple[tuple, ...]:
    """Give the m copies of a resampled source disjoint round-robin slices of its
    reservoir (copy j gets items j, j + m, ...), so no stored rollout is duplicated."""
    sel = np.asarray(list(selected), dtype=np.int64)
    if sel.size == 0:
        raise ValueError("partitioning needs at least one resampled index")
    if (sel < 0).any() or (sel >= len(reservoirs)).any():
        raise ValueError("resampled index outside the reservoir list")
    out: list[tuple] = [()] * sel.size
    for src in np.unique(sel):
        copies = np.flatnonzero(sel == src)
        items = list(reservoirs[int(src)])
        for j, dst in enumerate(copies):
            out[int(dst)] = tuple(items[j::copies.size])
    return tuple(out)
