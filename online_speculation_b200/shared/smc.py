"""Weight normalisation, systematic resampling and reservoir partitioning for SMC
(reference: src/inference_scaling/shared/smc.py:15-77)."""

from __future__ import annotations

from collections import defaultdict
from collections.abc import Sequence
from math import isfinite

import numpy as np


def normalize_smc_log_weights(log_weights: Sequence[float]) -> tuple[tuple[float, ...], float]:
    if not len(log_weights):
        raise ValueError("SMC requires at least one branch weight")
    v = np.asarray(log_weights, dtype=np.float64)
    if not np.all(np.isfinite(v)):
        raise ValueError("SMC log weights must be finite")
    w = np.exp(v - v.max())
    total = float(w.sum())
    if not isfinite(total) or total <= 0:
        raise ValueError("SMC weights cannot be normalized")
    p = w / total
    return tuple(float(x) for x in p), float(1.0 / np.square(p).sum())


def systematic_resample(probabilities: Sequence[float], count: int, generator: np.random.Generator) -> tuple[int, ...]:
    if count <= 0:
        raise ValueError("resampling count must be positive")
    p = np.asarray(probabilities, dtype=np.float64)
    if p.size == 0 or not np.all(np.isfinite(p)) or np.any(p < 0):
        raise ValueError("resampling probabilities must be finite and non-negative")
    total = float(p.sum())
    if total <= 0:
        raise ValueError("resampling probabilities must have positive mass")
    cdf = np.cumsum(p / total)
    cdf[-1] = 1.0
    points = float(generator.random()) / count + np.arange(count, dtype=np.float64) / count
    return tuple(int(i) for i in np.searchsorted(cdf, points, side="right"))


def partition_resampled_reservoirs(reservoirs: Sequence[Sequence], selected: Sequence[int]) -> tuple[tuple, ...]:
    """Split each source reservoir round-robin among its resampled copies (no duplication)."""
    if not len(selected):
        raise ValueError("at least one resampled index is required")
    if any(i < 0 or i >= len(reservoirs) for i in selected):
        raise ValueError("a resampled index lies outside the reservoir set")
    where: dict[int, list[int]] = defaultdict(list)
    for out, src in enumerate(selected):
        where[int(src)].append(out)
    outputs: list = [None] * len(selected)
    for src, outs in where.items():
        buckets = [[] for _ in outs]
        for i, item in enumerate(reservoirs[src]):
            buckets[i % len(buckets)].append(item)
        for o, b in zip(outs, buckets):
            outputs[o] = tuple(b)
    return tuple(outputs)
