"""Variance-cost optimal split of a rollout budget between history and fresh samples.

Problem (per candidate i with outer probability ratio r_i): estimate a mean
from n^h_i replayed history rollouts (std s^h_i, cost c^h_i each) and n^f_i
fresh rollouts (std s^f_i, cost c^f_i), minimising sum_i r_i^2 (s^2 / n) over
all sources subject to sum c n <= budget, n^h_i <= cap_i, per-group history
caps and a minimum number of fresh rollouts per candidate.  The Lagrangian
solution is n proportional to r s / sqrt(c); caps are handled by water
filling (a source whose share would exceed its cap is fixed at the cap and
the rest of the budget is re-split among the others), then counts are
rounded down and the leftover budget is given out by largest fractional
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


def _fill_capped(total: float, weights: np.ndarray, caps: np.ndarray) -> np.ndarray:
    """Split ``total`` proportionally to ``weights`` without exceeding ``caps`` (water filling)."""
    out = np.zeros_like(weights)
    free = weights > 0
    left = min(float(total), float(caps[free].sum()) if free.any() else 0.0)
    while left > 1e-12 and free.any():
        share = left * np.where(free, weights, 0.0) / weights[free].sum()
        over = free & (share >= caps - out - 1e-12)
        if not over.any():
            out += share
            break
        add = np.where(over, np.maximum(caps - out, 0.0), 0.0)
        out += add
        left -= float(add.sum())
        free &= ~over
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
    wh = np.array([ri * s.history_std / sqrt(s.history_cost) for ri, s in zip(r, statistics)])
    wf = np.array([ri * s.fresh_std / sqrt(s.fresh_cost) for ri, s in zip(r, statistics)])
    wh[hcap == 0] = 0.0
    budget = rollout_budget - float(minimum @ cf)
    if budget < -1e-9:
        raise ValueError("rollout budget cannot cover the required fresh sample for every candidate")
    hist = np.zeros(n)
    fresh = np.zeros(n)
    h_open = wh > 0
    groups = list(history_groups)
    g_left = {g: float(c) for g, c in group_capacities.items()}
    while budget > 1e-12:
        f_w = wf.copy()
        f_open = f_w > 0
        denom = float((wh * ch)[h_open].sum() + (f_w * cf)[f_open].sum())
        if denom <= 0:
            # no variance information: spread the remainder evenly over candidates that need fresh draws
            f_open = minimum > 0
            if not f_open.any():
                break
            f_w = 1.0 / cf
            denom = float((f_w * cf)[f_open].sum())
        ph = np.where(h_open, budget * wh / denom, 0.0)
        pf = np.where(f_open, budget * f_w / denom, 0.0)
        # a history group over its capacity: fix its members by capped proportional fill
        bad = next((g for g in dict.fromkeys(groups)
                    if sum(ph[i] for i in range(n) if h_open[i] and groups[i] == g) > g_left[g] + 1e-12), None)
        if bad is not None:
            members = [i for i in range(n) if h_open[i] and groups[i] == bad]
            fill = _fill_capped(g_left[bad], wh[members], hcap[members] - hist[members])
            cost = float(fill @ ch[members])
            if cost > budget + 1e-12:
                fill *= budget / cost
            for i, v in zip(members, fill):
                hist[i] += v
                budget -= v * ch[i]
                h_open[i] = False
            g_left[bad] = 0.0
            continue
        over = next((i for i in range(n) if h_open[i] and ph[i] > hcap[i] - hist[i] + 1e-12), None)
        if over is not None:
            add = hcap[over] - hist[over]
            hist[over] += add
            budget -= add * ch[over]
            g_left[groups[over]] = max(0.0, g_left[groups[over]] - add)
            h_open[over] = False
            continue
        hist += ph
        fresh += pf
        budget = 0.0
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
