"""RQMC rollout designs, exact bounded early stopping and the i-SIR kernel (CPU)."""

import math

import numpy as np
import pytest

from online_speculation_b200.arllm.algorithms.conditional_is import run_conditional_is
from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import ConditionalISConfig
from online_speculation_b200.experimental.shared.bounded_selection import invariant_categorical_index
from online_speculation_b200.experimental.shared.iterated_sir import (iterated_sir_transition,
                                                                       iterated_sir_tv_bound)
from online_speculation_b200.experimental.shared.rqmc import (randomized_lattice_uniforms,
                                                               scrambled_sobol_uniforms)
from online_speculation_b200.shared.rng import SeedStream
from online_speculation_b200.shared.stepwise import StepwiseCandidate, categorical_index_from_uniform


def _zeros(prompt, y):
    return sum(t == 0 for t in y) / len(y)


def test_lattice_points_are_evenly_spaced_and_marginally_uniform():
    pts = np.array(randomized_lattice_uniforms(8, seed=3))
    gaps = np.diff(np.sort(pts))
    assert np.allclose(gaps, 1 / 8)
    first = np.array([randomized_lattice_uniforms(4, seed=s)[2] for s in range(4000)])
    assert abs(first.mean() - 0.5) < 0.02 and abs((first < 0.25).mean() - 0.25) < 0.03


def test_sobol_net_is_stratified():
    pts = np.array(scrambled_sobol_uniforms(16, 3, seed=11))
    assert pts.shape == (16, 3) and np.all((pts >= 0) & (pts < 1))
    for d in range(3):   # a (0, m, s)-net: every 1/16 interval holds exactly one point per coordinate
        assert sorted(np.floor(pts[:, d] * 16).astype(int)) == list(range(16))


def test_invariant_index_holds_for_every_vector_in_the_box():
    rng = np.random.default_rng(0)
    hits = 0
    for _ in range(300):
        K = int(rng.integers(2, 6))
        lo = rng.uniform(0.1, 2.0, K)
        hi = lo + rng.uniform(0.0, 0.6, K) * rng.integers(0, 2, K)
        u = float(rng.random())
        idx = invariant_categorical_index(lo, hi, uniform=u)
        picks = {categorical_index_from_uniform(rng.uniform(lo, hi), u) for _ in range(200)}
        picks |= {categorical_index_from_uniform(lo, u), categorical_index_from_uniform(hi, u)}
        if idx is not None:
            hits += 1
            assert picks == {idx}
        if np.all(lo == hi):
            assert idx == categorical_index_from_uniform(lo, u)
    assert hits > 50


@pytest.mark.parametrize("design", ["scrambled_sobol", "arithmetic_lattice"])
def test_rqmc_conditional_is_targets_the_tilted_model(design):
    V, L, tau = 16, 8, 0.5
    backend = TabularBackend.per_position_logits(V, L, seed=5, prompt_length=1)
    cfg = ConditionalISConfig(candidate_count=6, rollout_count=4, block_size=2, total_length=L,
                              reward_temperature=tau, rollout_design=design)
    runs = [run_conditional_is(backend, (9,), cfg, _zeros, SeedStream(s)) for s in range(120)]
    p = backend.position_probabilities
    tilt = p[:, 0] * math.exp(1 / (L * tau))
    oracle = tilt / (tilt + 1 - p[:, 0])
    zeros = np.array([[r.token_ids[t] == 0 for t in range(L)] for r in runs], dtype=np.float64)
    assert abs(zeros.sum(1).mean() - oracle.sum()) < 0.45
    assert zeros.sum(1).mean() > p[:, 0].sum()
    with pytest.raises(ValueError):
        run_conditional_is(backend, (9,), cfg, seeds=SeedStream(0), reward_batch=lambda p, ys: [0.0] * len(ys))


def test_exact_early_stop_selects_what_full_evaluation_selects():
    V, L, tau = 12, 8, 0.5
    backend = TabularBackend.per_position_logits(V, L, seed=2, prompt_length=1)
    full = ConditionalISConfig(candidate_count=4, rollout_count=8, block_size=2, total_length=L,
                               reward_temperature=tau)
    bounded = ConditionalISConfig(candidate_count=4, rollout_count=8, block_size=2, total_length=L,
                                  reward_temperature=tau, exact_rollout_early_stop=True,
                                  rollout_log_weight_bounds=(0.0, 1.0 / tau), rollout_evaluation_batch_size=1)
    skipped = 0
    for s in range(12):
        a = run_conditional_is(backend, (3,), full, _zeros, SeedStream(s))
        b = run_conditional_is(backend, (3,), bounded, _zeros, SeedStream(s))
        assert a.token_ids == b.token_ids
        for st in b.steps:
            assert st.rollout_evaluations_performed + st.rollout_evaluations_skipped == st.rollout_evaluations_planned
            assert st.exact_early_stop == (st.rollout_evaluations_skipped > 0)
            for c in st.candidates:
                assert c.log_weight_lower_bound <= c.log_weight <= c.log_weight_upper_bound
            skipped += st.rollout_evaluations_skipped
    assert skipped > 0
    with pytest.raises(ValueError):
        ConditionalISConfig(exact_rollout_early_stop=True)
    narrow = ConditionalISConfig(candidate_count=2, rollout_count=2, block_size=2, total_length=4,
                                 reward_temperature=tau, exact_rollout_early_stop=True,
                                 rollout_log_weight_bounds=(0.0, 0.1))
    with pytest.raises(ValueError):
        run_conditional_is(backend, (3,), narrow, lambda p, y: 1.0, SeedStream(0))


def test_iterated_sir_is_invariant_on_a_finite_target():
    # target pi over 4 states, proposal q uniform; weight pi / q
    pi = np.array([0.1, 0.2, 0.3, 0.4])
    rng = np.random.default_rng(1)
    counts = np.zeros(4)
    state = StepwiseCandidate(0, math.log(pi[0] * 4))
    for it in range(20000):
        fresh = [StepwiseCandidate(int(x), math.log(pi[int(x)] * 4)) for x in rng.integers(0, 4, 2)]
        state = iterated_sir_transition(state, fresh, rng=rng).selected
        if it >= 100:
            counts[state.value] += 1
    assert np.allclose(counts / counts.sum(), pi, atol=0.02)
    assert iterated_sir_tv_bound(pool_size=3, updates=0, normalized_weight_supremum=1.6) == 1.0
    assert iterated_sir_tv_bound(pool_size=3, updates=5, normalized_weight_supremum=1.6) == pytest.approx(
        (1 - 2 / 4.2) ** 5)
