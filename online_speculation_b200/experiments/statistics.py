"""Estimators for experiment reports, vectorised over bootstrap replicates.

* Wilson score interval of a binomial proportion;
* the unbiased pass@k estimator 1 - C(n - c, k) / C(n, k);
* quantiles with linear interpolation between order statistics;
* percentile bootstrap of a mean (all replicates drawn as one index matrix);
* clustered paired bootstrap of a difference in success rates, resampling whole
  clusters (repeated draws of one problem stay together);
* total variation and Jensen-Shannon divergence (bits) between answer laws, and a
  bootstrap of their mean over problems.

Every bootstrap takes an explicit seed (numpy ``default_rng``), so reports are
reproducible.  The estimators are those of the reference's experiment reports
(experiments/shared/statistics.py); only their computation is different.
"""

from __future__ import annotations

import math
from collections.abc import Mapping, Sequence
from typing import Any

import numpy as np

from ..shared.metrics import total_variation

Z95 = 1.959963984540054


def wilson_interval(successes: int, trials: int, z: float = Z95) -> list[float]:
    if trials < 1 or not 0 <= successes <= trials:
        raise ValueError(f"need 0 <= successes <= trials and trials >= 1, got {successes}/{trials}")
    n = float(trials)
    p = successes / n
    shrink = 1.0 + z * z / n
    centre = (p + z * z / (2 * n)) / shrink
    spread = z * math.sqrt(p * (1 - p) / n + z * z / (4 * n * n)) / shrink
    return [centre - spread, centre + spread]


def estimated_pass_at_k(correct: int, draws: int, k: int) -> float:
    """Probability that k of the n draws, taken without replacement, include a correct one."""
    if not 0 <= correct <= draws:
        raise ValueError("correct must lie in 0..draws")
    if not 1 <= k <= draws:
        raise ValueError("k must lie in 1..draws")
    wrong = draws - correct
    if wrong < k:
        return 1.0
    # C(wrong, k) / C(draws, k) as a product of k ratios (no large integers)
    steps = np.arange(k, dtype=np.float64)
    ratio = np.prod((wrong - steps) / (draws - steps))
    return float(1.0 - ratio)


def quantile(values: Sequence[float], probability: float) -> float:
    if not len(values):
        raise ValueError("a quantile of no values is undefined")
    if not 0.0 <= probability <= 1.0:
        raise ValueError("probability must lie in [0, 1]")
    return float(np.quantile(np.asarray(values, dtype=np.float64), probability))


def _bootstrap_means(values: np.ndarray, seed: int, replicates: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    picks = rng.integers(0, values.size, size=(replicates, values.size))
    return values[picks].mean(axis=1)


def _central_95(samples: np.ndarray) -> list[float]:
    lo, hi = np.quantile(samples, [0.025, 0.975])
    return [float(lo), float(hi)]


def bootstrap_mean_interval(values: Sequence[float], *, seed: int, replicates: int = 10_000) -> list[float]:
    if not len(values) or replicates < 1:
        raise ValueError("the bootstrap needs values and a positive replicate count")
    return _central_95(_bootstrap_means(np.asarray(values, dtype=np.float64), seed, replicates))


def _rates_by_cluster(records: Sequence[Mapping[str, Any]], cluster_key: str, outcome_key: str
                      ) -> dict[int, np.ndarray]:
    grouped: dict[int, list[float]] = {}
    for record in records:
        grouped.setdefault(int(record[cluster_key]), []).append(float(bool(record[outcome_key])))
    return {c: np.asarray(v) for c, v in grouped.items()}


def clustered_paired_binary_difference(left_records: Sequence[Mapping[str, Any]],
                                       right_records: Sequence[Mapping[str, Any]], *, cluster_key: str,
                                       outcome_key: str, seed: int, replicates: int = 10_000) -> dict[str, Any]:
    """Mean over clusters of (left success rate - right success rate), with a cluster bootstrap interval."""
    if not left_records or not right_records or replicates < 1:
        raise ValueError("both methods need records, and the replicate count must be positive")
    left = _rates_by_cluster(left_records, cluster_key, outcome_key)
    right = _rates_by_cluster(right_records, cluster_key, outcome_key)
    if left.keys() != right.keys():
        raise ValueError("the two methods were not run on the same clusters")
    clusters = sorted(left)
    if any(left[c].size != right[c].size for c in clusters):
        raise ValueError("the two methods have different draw counts in some cluster")
    differences = np.asarray([left[c].mean() - right[c].mean() for c in clusters])
    return {"difference": float(differences.mean()),
            "clustered_bootstrap_95": _central_95(_bootstrap_means(differences, seed, replicates))}


def probability_distribution(counts: Mapping[str, int]) -> dict[str, float]:
    keys = list(counts)
    mass = np.asarray([counts[k] for k in keys], dtype=np.float64)
    if mass.sum() <= 0:
        raise ValueError("counts need positive total mass")
    return dict(zip(keys, (mass / mass.sum()).tolist()))


def total_variation_distance(left: Mapping[str, float], right: Mapping[str, float]) -> float:
    return total_variation(left, right)


def _aligned(left: Mapping[str, float], right: Mapping[str, float]) -> tuple[np.ndarray, np.ndarray]:
    keys = sorted(set(left) | set(right), key=str)
    return (np.asarray([left.get(k, 0.0) for k in keys], dtype=np.float64),
            np.asarray([right.get(k, 0.0) for k in keys], dtype=np.float64))


def jensen_shannon_bits(left: Mapping[str, float], right: Mapping[str, float]) -> float:
    p, q = _aligned(left, right)
    m = 0.5 * (p + q)

    def kl_to_mid(a: np.ndarray) -> float:
        support = a > 0
        return float(np.sum(a[support] * np.log2(a[support] / m[support])))

    return 0.5 * (kl_to_mid(p) + kl_to_mid(q))


def bootstrap_answer_distance(left: Mapping[int, Sequence[str]], right: Mapping[int, Sequence[str]],
                              problem_indices: Sequence[int], *, seed: int = 0,
                              replicates: int = 2_000) -> dict[str, list[float]]:
    """Bootstrap of the mean (over problems) TV and JS distance between two methods' answers."""
    if not problem_indices or replicates < 1:
        raise ValueError("the bootstrap needs problems and a positive replicate count")
    rng = np.random.default_rng(seed)
    tv = np.zeros(replicates)
    js = np.zeros(replicates)
    for i in problem_indices:
        a, b = list(left[i]), list(right[i])
        if not a or not b:
            raise ValueError(f"problem {i} lacks answers from one of the methods")
        labels = sorted(set(a) | set(b), key=str)
        code = {label: j for j, label in enumerate(labels)}
        ca, cb = np.asarray([code[x] for x in a]), np.asarray([code[x] for x in b])
        ra = ca[rng.integers(0, ca.size, size=(replicates, ca.size))]
        rb = cb[rng.integers(0, cb.size, size=(replicates, cb.size))]
        pa = np.stack([np.bincount(r, minlength=len(labels)) for r in ra]) / ca.size
        pb = np.stack([np.bincount(r, minlength=len(labels)) for r in rb]) / cb.size
        tv += 0.5 * np.abs(pa - pb).sum(axis=1)
        m = 0.5 * (pa + pb)
        with np.errstate(divide="ignore", invalid="ignore"):
            kl_a = np.where(pa > 0, pa * np.log2(pa / m), 0.0).sum(axis=1)
            kl_b = np.where(pb > 0, pb * np.log2(pb / m), 0.0).sum(axis=1)
        js += 0.5 * (kl_a + kl_b)
    tv /= len(problem_indices)
    js /= len(problem_indices)
    return {"mean_total_variation_bootstrap_95": _central_95(tv),
            "mean_jensen_shannon_bits_bootstrap_95": _central_95(js)}


__all__ = ["bootstrap_answer_distance", "bootstrap_mean_interval", "clustered_paired_binary_difference",
           "estimated_pass_at_k", "jensen_shannon_bits", "probability_distribution", "quantile",
           "total_variation_distance", "wilson_interval"]
