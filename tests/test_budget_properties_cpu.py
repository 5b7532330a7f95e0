"""Property tests (hypothesis) of the variance-cost budget allocator: hard constraints of the integer
allocation, and the optimality conditions of its continuous solution (equal marginal variance
reduction per unit cost among unconstrained sources, capped sources wanting more)."""

import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st

from online_speculation_b200.shared.budget import VarianceCostEstimate, allocate_variance_cost_budget

positive = st.floats(min_value=0.1, max_value=5.0, allow_nan=False, allow_infinity=False)


@st.composite
def instances(draw):
    n = draw(st.integers(1, 5))
    ratios = [draw(positive) for _ in range(n)]
    stats = [VarianceCostEstimate(draw(positive), draw(positive), draw(positive), draw(positive)) for _ in range(n)]
    caps = [draw(st.integers(0, 6)) for _ in range(n)]
    groups = [draw(st.integers(0, 1)) for _ in range(n)]
    group_caps = {0: draw(st.integers(0, 8)), 1: draw(st.integers(0, 8))}
    minimum = [draw(st.integers(0, 2)) for _ in range(n)]
    floor = sum(m * s.fresh_cost for m, s in zip(minimum, stats))
    budget = floor + draw(st.floats(min_value=0.5, max_value=40.0))
    return ratios, stats, caps, groups, group_caps, minimum, budget


@settings(max_examples=300, deadline=None)
@given(instances())
def test_allocation_properties(inst):
    ratios, stats, caps, groups, group_caps, minimum, budget = inst
    alloc = allocate_variance_cost_budget(outer_ratios=ratios, statistics=stats, history_capacities=caps,
                                          history_groups=groups, group_capacities=group_caps, rollout_budget=budget,
                                          minimum_fresh=minimum)
    n = len(ratios)
    hist = np.array([a.history_count for a in alloc])
    fresh = np.array([a.fresh_count for a in alloc])
    ch = np.array([s.history_cost for s in stats])
    cf = np.array([s.fresh_cost for s in stats])
    # integer allocation: every hard constraint
    assert (hist >= 0).all() and (hist <= np.array(caps)).all()
    assert (fresh >= np.array(minimum)).all()
    for g in (0, 1):
        assert hist[[i for i in range(n) if groups[i] == g]].sum() <= group_caps[g]
    assert float(hist @ ch + fresh @ cf) <= budget + 1e-6
    # continuous solution: feasible, and optimal by its first-order conditions
    ch_n = np.array([a.continuous_history for a in alloc])
    cf_n = np.array([a.continuous_fresh for a in alloc]) - np.array(minimum)
    assert (ch_n >= -1e-9).all() and (ch_n <= np.array(caps) + 1e-6).all() and (cf_n >= -1e-9).all()
    spent = float(ch_n @ ch + (cf_n + np.array(minimum)) @ cf)
    assert spent <= budget + 1e-6
    # weight of a source: r s / sqrt(c); an interior optimum sets n proportional to it at one common
    # multiplier (n / weight equal), a source held at its cap would take more (n / weight below it)
    wh = np.array([r * s.history_std / np.sqrt(s.history_cost) for r, s in zip(ratios, stats)])
    wf = np.array([r * s.fresh_std / np.sqrt(s.fresh_cost) for r, s in zip(ratios, stats)])
    free_fresh = [cf_n[i] / wf[i] for i in range(n) if wf[i] > 0]
    assert len(free_fresh) == n
    level = free_fresh[0]
    assert np.allclose(free_fresh, level, rtol=1e-6, atol=1e-9)    # fresh draws are never capped
    gcap_full = {g: ch_n[[i for i in range(n) if groups[i] == g]].sum() >= group_caps[g] - 1e-6 for g in (0, 1)}
    for i in range(n):
        if caps[i] == 0 or wh[i] == 0:
            assert ch_n[i] <= 1e-9
            continue
        ratio = ch_n[i] / wh[i]
        at_cap = ch_n[i] >= caps[i] - 1e-6 or gcap_full[groups[i]]
        if at_cap:
            assert ratio <= level * (1 + 1e-6) + 1e-9
        else:
            assert np.isclose(ratio, level, rtol=1e-6, atol=1e-9)
    # with uncapped fresh sources the whole budget is spent
    assert spent >= budget - 1e-6


def test_a_group_cap_that_does_not_bind_leaves_members_at_their_optimum():
    # one member's share exceeds its own cap; the group (capacity 3) is not full at the optimum:
    # h1 = 1 (its cap), then lambda re-prices the rest: h2 = 9 * w2 / (3 + 2 w2) with w2 = 1 / sqrt(2)
    stats = [VarianceCostEstimate(1, 1, 1, 1), VarianceCostEstimate(1, 1, 1, 1), VarianceCostEstimate(1, 1, 2, 1)]
    a = allocate_variance_cost_budget(outer_ratios=[1, 1, 1], statistics=stats, history_capacities=[0, 1, 2],
                                      history_groups=[0, 0, 0], group_capacities={0: 3}, rollout_budget=10.0,
                                      minimum_fresh=0)
    w2 = 1 / np.sqrt(2)
    assert a[1].continuous_history == np.float64(1.0) or abs(a[1].continuous_history - 1.0) < 1e-9
    assert abs(a[2].continuous_history - 9 * w2 / (3 + 2 * w2)) < 1e-6
    assert all(abs(x.continuous_fresh - 9 / (3 + 2 * w2)) < 1e-6 for x in a)
