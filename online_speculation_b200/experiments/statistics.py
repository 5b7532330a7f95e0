"""Estimators used by experiment reports (model independent).

Wilson score intervals, the unbiased pass@k estimator, linear-interpolation
quantiles, percentile bootstrap of a mean, a clustered paired bootstrap of a
binary difference (repeated draws per problem kept together), total variation
and Jensen-Shannon divergence (bits) between answer distributions, and a
bootstrap of the mean distance between two methods' answer distributions.

Reference behaviour: experiments/shared/statistics.py:14-206.
"""

from __future__ import annotations

import math
import random
from collections import Counter
from collections.abc import Mapping, Sequence
from statistics import fmean
from typing import Any

from ..shared.metrics import total_variation

Z95 = 1.959963984540054


def wilson_interval(successes: int, trials: int, z: float = Z95) -> list[float]:
    if trials <= 0 or not 0 <= successes <= trials:
        raise ValueError("successes must lie between zero and positive trials")
    p = successes / trials
    zz = z * z
    den = 1.0 + zz / trials
    centre = (p + zz / (2 * trials)) / den
    half = z * math.sqrt(p * (1 - p) / trials + zz / (4 * trials * trials)) / den
    return [centre - half, centre + half]


def estimated_pass_at_k(correct: int, draws: int, k: int) -> float:
    """1 - C(n - c, k) / C(n, k): probability that k draws without replacement contain a correct one."""
    if not 0 <= correct <= draws:
        raise ValueError("correct must lie between zero and draws")
    if draws <= 0 or not 1 <= k <= draws:
        raise ValueError("k must lie between one and the number of draws")
    if draws - correct < k:
        return 1.0
    return 1.0 - math.comb(draws - correct, k) / math.comb(draws, k)


def quantile(values: Sequence[float], probability: float) -> float:
    if not len(values):
        raise ValueError("quantile requires at least one value")
    if not 0 <= probability <= 1:
        raise ValueError("probability must lie in [0, 1]")
    v = sorted(float(x) for x in values)
    pos = (len(v) - 1) * probability
    lo, hi = math.floor(pos), math.ceil(pos)
    return v[lo] if lo == hi else v[lo] + (v[hi] - v[lo]) * (pos - lo)


def _resample_means(values: Sequence[float], rng: random.Random, replicates: int) -> list[float]:
    n = len(values)
    return [fmean(values[rng.randrange(n)] for _ in range(n)) for _ in range(replicates)]


def bootstrap_mean_interval(values: Sequence[float], *, seed: int, replicates: int = 10_000) -> list[float]:
    if not len(values) or replicates <= 0:
        raise ValueError("bootstrap values and replicate count must be positive")
    means = _resample_means([float(x) for x in values], random.Random(seed), replicates)
    return [quantile(means, 0.025), quantile(means, 0.975)]


def clustered_paired_binary_difference(left_records: Sequence[Mapping[str, Any]],
                                       right_records: Sequence[Mapping[str, Any]], *, cluster_key: str,
                                       outcome_key: str, seed: int, replicates: int = 10_000) -> dict[str, Any]:
    """Mean over clusters of (left success rate - right success rate), with a cluster bootstrap interval."""
    if not left_records or not right_records or replicates <= 0:
        raise ValueError("paired records and replicate count must be positive")

    def by_cluster(records):
        out: dict[int, list[float]] = {}
        for r in records:
            out.setdefault(int(r[cluster_key]), []).append(float(bool(r[outcome_key])))
        return out

    left, right = by_cluster(left_records), by_cluster(right_records)
    if left.keys() != right.keys():
        raise ValueError("paired methods must contain the same clusters")
    diffs = []
    for c in sorted(left):
        if len(left[c]) != len(right[c]):
            raise ValueError("paired methods must contain the same draws per cluster")
        diffs.append(fmean(left[c]) - fmean(right[c]))
    boot = _resample_means(diffs, random.Random(seed), replicates)
    return {"difference": fmean(diffs), "clustered_bootstrap_95": [quantile(boot, 0.025), quantile(boot, 0.975)]}


def probability_distribution(counts: Mapping[str, int]) -> dict[str, float]:
    total = sum(counts.values())
    if total <= 0:
        raise ValueError("counts must have positive mass")
    return {k: v / total for k, v in counts.items()}


def total_variation_distance(left: Mapping[str, float], right: Mapping[str, float]) -> float:
    return total_variation(left, right)


def jensen_shannon_bits(left: Mapping[str, float], right: Mapping[str, float]) -> float:
    keys = set(left) | set(right)
    mid = {k: 0.5 * (left.get(k, 0.0) + right.get(k, 0.0)) for k in keys}

    def kl(d):
        return sum(p * math.log2(p / mid[k]) for k, p in d.items() if p > 0)

    return 0.5 * (kl(left) + kl(right))


def bootstrap_answer_distance(left: Mapping[int, Sequence[str]], right: Mapping[int, Sequence[str]],
                              problem_indices: Sequence[int], *, seed: int = 0,
                              replicates: int = 2_000) -> dict[str, list[float]]:
    if not problem_indices or replicates <= 0:
        raise ValueError("problem indices and replicate count must be positive")
    rng = random.Random(seed)
    tv, js = [], []
    for _ in range(replicates):
        t_sum, j_sum = 0.0, 0.0
        for i in problem_indices:
            a, b = left[i], right[i]
            if not a or not b:
                raise ValueError("every problem requires observations from both methods")
            pa = probability_distribution(Counter(a[rng.randrange(len(a))] for _ in a))
            pb = probability_distribution(Counter(b[rng.randrange(len(b))] for _ in b))
            t_sum += total_variation_distance(pa, pb)
            j_sum += jensen_shannon_bits(pa, pb)
        tv.append(t_sum / len(problem_indices))
        js.append(j_sum / len(problem_indices))
    return {"mean_total_variation_bootstrap_95": [quantile(tv, 0.025), quantile(tv, 0.975)],
            "mean_jensen_shannon_bits_bootstrap_95": [quantile(js, 0.025), quantile(js, 0.975)]}


__all__ = ["bootstrap_answer_distance", "bootstrap_mean_interval", "clustered_paired_binary_difference",
           "estimated_pass_at_k", "jensen_shannon_bits", "probability_distribution", "quantile",
           "total_variation_distance", "wilson_interval"]
