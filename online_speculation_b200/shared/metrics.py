"""Distribution and sampling diagnostics (reference: src/inference_scaling/shared/metrics.py)."""

from __future__ import annotations

from collections import Counter
from collections.abc import Iterable, Mapping, Sequence
from math import fsum

import numpy as np


def normalize_counts(counts: Mapping) -> dict:
    total = sum(counts.values())
    if total == 0:
        raise ValueError("at least one sample is required")
    return {k: c / total for k, c in counts.items()}


def empirical_distribution(samples: Iterable) -> dict:
    return normalize_counts(Counter(samples))


def total_variation(left: Mapping, right: Mapping) -> float:
    return 0.5 * fsum(abs(left.get(k, 0.0) - right.get(k, 0.0)) for k in set(left) | set(right))


def importance_effective_sample_size(log_weights: Sequence[float]) -> float:
    if not len(log_weights):
        return 0.0
    values = np.asarray(log_weights, dtype=np.float64)
    top = float(values.max())
    if not np.isfinite(top):
        return 0.0
    w = np.exp(values - top)
    den = float(w @ w)
    return float(w.sum() ** 2 / den) if den > 0 else 0.0


def autocorrelation_ess(values: Sequence[float]) -> float:
    """Initial-positive-sequence estimate of a Markov chain's effective sample size."""
    x = np.asarray(values, dtype=np.float64)
    n = x.size
    if n < 2:
        return float(n)
    c = x - x.mean()
    var = float(c @ c / n)
    if var == 0:
        return float(n)
    rho: list[float] = []
    for lag in range(1, n):
        r = float(c[:-lag] @ c[lag:] / (n - lag)) / var
        if lag % 2 == 0 and rho and rho[-1] + r <= 0:
            break
        rho.append(r)
    tau = max(1.0, 1.0 + 2.0 * sum(rho))
    return min(float(n), n / tau)
