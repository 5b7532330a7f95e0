"""Property tests (hypothesis) of the sampling primitives: MH acceptance and detailed balance,
inverse-CDF categorical draws, bounded-weight selection, effective sample sizes, RQMC uniforms."""

import itertools
import math

import numpy as np
import pytest
from hypothesis import assume, given, settings
from hypothesis import strategies as st

from online_speculation_b200.experimental.shared.bounded_selection import invariant_categorical_index
from online_speculation_b200.experimental.shared.rqmc import randomized_lattice_uniforms, scrambled_sobol_uniforms
from online_speculation_b200.shared.metrics import autocorrelation_ess, importance_effective_sample_size
from online_speculation_b200.shared.mh import decide_metropolis_hastings, mh_log_acceptance_batch
from online_speculation_b200.shared.stepwise import categorical_index_from_uniform

finite = st.floats(min_value=-30, max_value=30, allow_nan=False)
unit = st.floats(min_value=0.0, max_value=1.0, exclude_max=True, allow_nan=False)


@settings(max_examples=300, deadline=None)
@given(finite, finite, finite, finite, unit)
def test_mh_acceptance_is_min_one_hastings_ratio(cur, prop, fwd, rev, u):
    d = decide_metropolis_hastings(current_target_log_density=cur, proposed_target_log_density=prop, uniform=u,
                                   forward_proposal_log_probability=fwd, reverse_proposal_log_probability=rev)
    ratio = (prop - cur) + (rev - fwd)
    assert d.log_acceptance == pytest.approx(min(0.0, ratio), abs=1e-12)
    assert 0.0 <= d.acceptance_probability <= 1.0
    assert d.accepted == (math.log(max(u, np.finfo(float).tiny)) <= min(0.0, ratio))


@settings(max_examples=60, deadline=None)
@given(st.lists(st.floats(min_value=0.05, max_value=5.0), min_size=2, max_size=5),
       st.lists(st.floats(min_value=0.05, max_value=5.0), min_size=2, max_size=5))
def test_mh_kernel_satisfies_detailed_balance(target_w, prop_w):
    """The MH kernel built from the acceptance rule leaves the target invariant (exact matrices)."""
    n = min(len(target_w), len(prop_w))
    pi = np.asarray(target_w[:n]) / sum(target_w[:n])
    q = np.asarray(prop_w[:n]) / sum(prop_w[:n])           # independence proposal
    K = np.zeros((n, n))
    for x, y in itertools.product(range(n), repeat=2):
        if x != y:
            a = math.exp(float(mh_log_acceptance_batch(math.log(pi[x]), math.log(pi[y]), math.log(q[y]),
                                                       math.log(q[x]))))
            K[x, y] = q[y] * a
    K[np.diag_indices(n)] = 1 - K.sum(1)
    flow = pi[:, None] * K
    assert np.allclose(flow, flow.T, atol=1e-12)
    assert np.allclose(pi @ K, pi, atol=1e-12)


@settings(max_examples=300, deadline=None)
@given(st.lists(st.floats(min_value=0.0, max_value=10.0), min_size=1, max_size=8), unit)
def test_categorical_draw_lands_in_its_cdf_interval(weights, u):
    assume(sum(weights) > 1e-6)
    i = categorical_index_from_uniform(weights, u)
    cdf = np.cumsum(np.asarray(weights) / sum(weights))
    lo = cdf[i - 1] if i else 0.0
    assert weights[i] > 0 and lo <= u + 1e-12 and (u < cdf[i] + 1e-12 or i == len(weights) - 1)


def test_categorical_draws_follow_the_law():
    p = np.array([0.1, 0.0, 0.6, 0.3])
    grid = (np.arange(100000) + 0.5) / 100000
    counts = np.bincount([categorical_index_from_uniform(p, u) for u in grid], minlength=4) / grid.size
    assert np.allclose(counts, p, atol=1e-4)


@settings(max_examples=300, deadline=None)
@given(st.lists(st.tuples(st.floats(min_value=0.1, max_value=5.0), st.floats(min_value=0.0, max_value=2.0)),
                min_size=1, max_size=6), unit, st.floats(min_value=0.0, max_value=1.0))
def test_bounded_selection_agrees_with_every_weight_in_the_box(boxes, u, t):
    lo = [a for a, _ in boxes]
    hi = [a + w for a, w in boxes]
    i = invariant_categorical_index(lo, hi, uniform=u)
    if i is None:
        return
    # any weight vector inside the box (here: corners mixed by t, and the two extreme corners) picks i
    for w in (lo, hi, [a + t * (b - a) for a, b in zip(lo, hi)]):
        assert categorical_index_from_uniform(w, u) == i


@settings(max_examples=200, deadline=None)
@given(st.lists(finite, min_size=1, max_size=20), st.floats(min_value=-50, max_value=50))
def test_importance_ess_bounds_and_shift_invariance(logw, shift):
    e = importance_effective_sample_size(logw)
    assert 1.0 - 1e-9 <= e <= len(logw) + 1e-9
    assert importance_effective_sample_size([v + shift for v in logw]) == pytest.approx(e, rel=1e-9)
    assert importance_effective_sample_size([0.0] * len(logw)) == pytest.approx(len(logw))


def test_autocorrelation_ess_orders_chains():
    rng = np.random.default_rng(0)
    iid = rng.normal(size=4000)
    ar = np.zeros(4000)
    for t in range(1, 4000):
        ar[t] = 0.9 * ar[t - 1] + rng.normal()
    e_iid, e_ar = autocorrelation_ess(iid), autocorrelation_ess(ar)
    assert 3000 < e_iid <= 4000
    # AR(1) with phi = 0.9: integrated time (1 + phi) / (1 - phi) = 19
    assert 4000 / 30 < e_ar < 4000 / 12


def test_rqmc_uniforms_are_uniform_and_stratified():
    lat = np.asarray(randomized_lattice_uniforms(64, seed=3))
    assert lat.min() >= 0 and lat.max() < 1
    # one point per stratum of width 1/64
    assert sorted(np.floor(lat * 64).astype(int).tolist()) == list(range(64))
    sob = np.asarray(scrambled_sobol_uniforms(256, 3, seed=5))
    assert sob.shape == (256, 3) and sob.min() >= 0 and sob.max() < 1
    for d in range(3):
        assert sorted(np.floor(sob[:, d] * 256).astype(int).tolist()) == list(range(256))
    means = np.mean([np.asarray(randomized_lattice_uniforms(16, seed=s)).mean() for s in range(400)])
    assert abs(means - 0.5) < 0.01
