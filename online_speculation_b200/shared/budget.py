"""Variance-cost optimal split of a rollout budget between history and fresh samples.

Problem (per candidate i with outer probability ratio r_i): estimate a mean
from n^h_i replayed history rollouts (std s^h_i, cost c^h_i each) and n^f_i
fresh rollouts (std s^f_i, cost c^f_i), minimising sum over all sources of
a / n with a = (r s)^2, subject to sum c n <= budget, n^h_i <= cap_i, per-group
history caps and a minimum number of fresh rollouts per candidate.  The problem
is convex and separable, so its optimum is the KKT point
n = min(cap, sqrt(a / (lambda c + mu_g))): lambda prices the budget, mu_g >= 0
the history group g (zero unless the group is full), fresh sources have no cap.
Both multipliers are found by bisection -- each group's mu for a given lambda,
lambda for the budget -- so the continuous solution is exact to rounding.
Without any cap binding this is n proportional to r s / sqrt(c).  Counts are
then rounded down and the leftover budget is given out by largest fractional
remainder while every hard constraint still holds.

Reference behaviour: src/inference_scaling/shared/budget.py:46-353.
"""

from __future__ import annotations

from collections.abc import Hashable, Mapping, Sequence
from dataclasses import dataclass
from math import isfinite, sqrt

import numpy as np


@dataclass(frozen=True, slots=True)
class VarianceCostEstimate:
    history_std: float
    fresh_std: float
    history_cost: float = 1.0
    fresh_cost: float = 1.0

    def __post_init__(self) -> None:
        vals = (self.history_std, self.fresh_std, self.history_cost, self.fresh_cost)
        if not all(isfinite(v) for v in vals):
            raise ValueError("variance and cost estimates must be finite")
        if self.history_std < 0 or self.fresh_std < 0:
            raise ValueError("standard deviations must be non-negative")
        if self.history_cost <= 0 or self.fresh_cost <= 0:
            raise ValueError("per-sample costs must be positive")


@dataclass(frozen=True, slots=True)
class BudgetAllocation:
    history_count: int
    fresh_count: int
    continuous_history: float
    continuous_fresh: float
    estimated_cost: float


def allocate_fresh_rollout_budget(*, outer_ratios: Sequence[float], standard_deviations: Sequence[float],
                                  costs: Sequence[float], rollout_budget: float,
                                  minimum_fresh: int | Sequence[int] = 1) -> tuple[BudgetAllocation, ...]:
    """The allocator restricted to fresh rollouts (no history)."""
    n = len(outer_ratios)
    if len(standard_deviations) != n or len(costs) != n:
        raise ValueError("fresh allocation inputs must have the same length")
    return allocate_variance_cost_budget(
        outer_ratios=outer_ratios,
        statistics=[VarianceCostEstimate(0.0, s, fresh_cost=c) for s, c in zip(standard_deviations, costs)],
        history_capacities=[0] * n, history_groups=list(range(n)), group_capacities={i: 0 for i in range(n)},
        rollout_budget=rollout_budget, minimum_fresh=minimum_fresh)


def _bisect(fn, target: float, lo: float, hi: float, iterations: int = 200) -> float:
    """The smallest argument (to rounding) where a non-increasing ``fn`` is at most ``target``
    (geometric bisection; ``hi`` grows until it brackets the crossing)."""
    if fn(lo) <= target:
        return lo
    for _ in range(400):
        if fn(hi) <= target:
            break
        hi *= 4.0
    for _ in range(iterations):
        mid = sqrt(lo * hi)
        if fn(mid) > target:
            lo = mid
        else:
            hi = mid
        if hi <= lo * (1 + 1e-15):
            break
    return hi


def _history_at(lam: float, a: np.ndarray, c: np.ndarray, cap: np.ndarray, groups: list, room: Mapping) -> np.ndarray:
    """History counts at budget price ``lam``: per group the smallest mu >= 0 that keeps it within its room."""
    out = np.zeros_like(a)
    for g in dict.fromkeys(groups):
        idx = np.asarray([i for i, gi in enumerate(groups) if gi == g and a[i] > 0 and cap[i] > 0], dtype=np.int64)
        if idx.size == 0:
            continue

        def counts(mu, idx=idx):
            return np.minimum(cap[idx], np.sqrt(a[idx] / (lam * c[idx] + mu)))

        total = float(room[g])
        if counts(0.0).sum() <= total:
            out[idx] = counts(0.0)
        elif total <= 0:
            out[idx] = 0.0
        else:
            hi = max(1.0, float((a[idx] / np.maximum(total / idx.size, 1e-300) ** 2).max()))
            mu = _bisect(lambda m: float(counts(m).sum()), total, 1e-300, hi * 4)
            out[idx] = counts(mu)
    return out


def allocate_variance_cost_budget(*, outer_ratios: Sequence[float], statistics: Sequence[VarianceCostEstimate],
                                  history_capacities: Sequence[int], history_groups: Sequence[Hashable],
                                  group_capacities: Mapping[Hashable, int], rollout_budget: float,
                                  minimum_fresh: int | Sequence[int] = 1) -> tuple[BudgetAllocation, ...]:
    n = len(outer_ratios)
    if n == 0:
        raise ValueError("at least one candidate is required")
    if not (len(statistics) == n == len(history_capacities) == len(history_groups)):
        raise ValueError("all candidate-level allocation inputs must have the same length")
    if not (rollout_budget > 0 and isfinite(rollout_budget)):
        raise ValueError("rollout_budget must be positive and finite")
    minimum = np.full(n, minimum_fresh, dtype=np.int64) if isinstance(minimum_fresh, int) else np.asarray(
        minimum_fresh, dtype=np.int64)
    if minimum.shape != (n,):
        raise ValueError("minimum_fresh must have one value per candidate")
    if (minimum < 0).any():
        raise ValueError("minimum fresh counts must be non-negative")
    r = np.asarray(outer_ratios, dtype=np.float64)
    if not np.isfinite(r).all() or (r <= 0).any():
        raise ValueError("outer probability ratios must be positive and finite")
    hcap = np.asarray(history_capacities, dtype=np.float64)
    if (hcap < 0).any():
        raise ValueError("history capacities must be non-negative")
    missing = set(history_groups) - set(group_capacities)
    if missing:
        raise ValueError(f"history groups are missing capacities: {sorted(map(repr, missing))}")
    if any(v < 0 for v in group_capacities.values()):
        raise ValueError("history group capacities must be non-negative")
    ch = np.array([s.history_cost for s in statistics])
    cf = np.array([s.fresh_cost for s in statistics])
    budget = rollout_budget - float(minimum @ cf)
    if budget < -1e-9:
        raise ValueError("rollout budget cannot cover the required fresh sample for every candidate")
    groups = list(history_groups)
    ah = np.where(hcap > 0, (r * np.array([s.history_std for s in statistics])) ** 2, 0.0)
    af = (r * np.array([s.fresh_std for s in statistics])) ** 2
    room = {g: float(c) for g, c in group_capacities.items()}
    hist = np.zeros(n)
    fresh = np.zeros(n)
    if budget > 1e-12:
        if (af > 0).any():
            def spend(lam):
                h = _history_at(lam, ah, ch, hcap, groups, room)
                f = np.sqrt(af / (lam * cf))
                return float(h @ ch + f @ cf)

            # a price high enough that almost nothing is bought, and one low enough to overspend
            hi_p = max(1.0, float(((ah + af) / np.minimum(ch, cf) / (budget / n) ** 2).max()) * 4)
            lam = _bisect(spend, budget, 1e-300, hi_p)
            hist = _history_at(lam, ah, ch, hcap, groups, room)
            fresh = np.sqrt(af / (lam * cf))
            scale = budget / max(float(hist @ ch + fresh @ cf), 1e-300)
            if scale < 1:           # the bisection lands on the feasible side; absorb its last bit
                hist *= scale
                fresh *= scale
        elif (ah > 0).any():
            # no fresh variance: history only, capped (the rest of the budget stays unspent)
            def spend_h(lam):
                return float(_history_at(lam, ah, ch, hcap, groups, room) @ ch)

            if spend_h(1e-300) <= budget:
                hist = _history_at(1e-300, ah, ch, hcap, groups, room)
            else:
                hi_p = max(1.0, float((ah / ch / (budget / n) ** 2).max()) * 4)
                hist = _history_at(_bisect(spend_h, budget, 1e-300, hi_p), ah, ch, hcap, groups, room)
        else:
            # no variance information: spread the remainder evenly over candidates that need fresh draws
            need = minimum > 0
            if need.any():
                fresh = np.where(need, budget / float(cf[need].sum()), 0.0)
    cont_f = minimum + fresh
    hi = np.floor(hist + 1e-12).astype(np.int64)
    fi = minimum + np.floor(fresh + 1e-12).astype(np.int64)
    left = rollout_budget - float(hi @ ch + fi @ cf)
    used: dict = {}
    for i, g in enumerate(groups):
        used[g] = used.get(g, 0) + int(hi[i])
    rema = [(float(hist[i] - hi[i]), i, "history") for i in range(n) if hist[i] - hi[i] > 1e-12]
    rema += [(float(cont_f[i] - fi[i]), i, "fresh") for i in range(n) if cont_f[i] - fi[i] > 1e-12]
    for _, i, src in sorted(rema, key=lambda t: (-t[0], t[1], t[2])):
        cost = ch[i] if src == "history" else cf[i]
        if cost > left + 1e-9:
            continue
        if src == "history":
            if hi[i] >= hcap[i] or used.get(groups[i], 0) >= group_capacities[groups[i]]:
                continue
            hi[i] += 1
            used[groups[i]] = used.get(groups[i], 0) + 1
        else:
            fi[i] += 1
        left -= float(cost)
    return tuple(BudgetAllocation(int(hi[i]), int(fi[i]), float(hist[i]), float(cont_f[i]),
                                  float(hi[i] * ch[i] + fi[i] * cf[i])) for i in range(n))


__all__ = ["BudgetAllocation", "VarianceCostEstimate", "allocate_fresh_rollout_budget",
           "allocate_variance_cost_budget"]
