"""Sampling diagnostics: empirical laws, total variation and effective sample sizes.

* importance ESS in log space: ESS = exp(2 LSE(v) - LSE(2 v)), which equals
  (sum w)^2 / sum w^2 for w = exp(v) without forming the weights;
* Markov-chain ESS from Geyer's initial positive sequence: autocorrelations come
  from one FFT of the centred series, consecutive pairs rho_{2k} + rho_{2k+1}
  are summed while positive, and tau = -1 + 2 * (that sum).

The function names follow src/inference_scaling/shared/metrics.py.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Iterable, Mapping, Sequence

import numpy as np


def normalize_counts(counts: Mapping) -> dict:
    keys = list(counts)
    mass = np.asarray([counts[k] for k in keys], dtype=np.float64)
    if mass.sum() == 0:
        raise ValueError("an empirical distribution needs at least one sample")
    return dict(zip(keys, (mass / mass.sum()).tolist()))


def empirical_distribution(samples: Iterable) -> dict:
    return normalize_counts(Counter(samples))


def total_variation(left: Mapping, right: Mapping) -> float:
    support = list(set(left) | set(right))
    a = np.asarray([left.get(k, 0.0) for k in support], dtype=np.float64)
    b = np.asarray([right.get(k, 0.0) for k in support], dtype=np.float64)
    return float(0.5 * np.abs(a - b).sum())


def _lse(v: np.ndarray) -> float:
    top = float(v.max())
    return top + float(np.log(np.exp(v - top).sum()))


def importance_effective_sample_size(log_weights: Sequence[float]) -> float:
    v = np.asarray(list(log_weights), dtype=np.float64)
    if v.size == 0 or not np.isfinite(v.max()):
        return 0.0
    return float(np.exp(2.0 * _lse(v) - _lse(2.0 * v)))


def autocorrelation_ess(values: Sequence[float]) -> float:
    """Effective sample size of a scalar Markov-chain trace (Geyer's initial positive sequence)."""
    x = np.asarray(list(values), dtype=np.float64)
    n = x.size
    if n < 2:
        return float(n)
    c = x - x.mean()
    if not np.any(c):
        return float(n)
    size = 1 << (2 * n - 1).bit_length()
    f = np.fft.rfft(c, size)
    acov = np.fft.irfft(f * np.conj(f), size)[:n] / np.arange(n, 0, -1)
    rho = acov / acov[0]
    pairs = rho[: n - n % 2].reshape(-1, 2).sum(1)
    positive = np.flatnonzero(pairs <= 0.0)
    kept = pairs[: positive[0]] if positive.size else pairs
    tau = max(1.0, -1.0 + 2.0 * float(kept.sum()))
    return min(float(n), n / tau)
