"""Distributional acceptance tests of the algorithm layer against exact oracles (CPU)."""

import itertools
import math

import numpy as np
import pytest

from online_speculation_b200.arllm.algorithms.conditional_is import run_conditional_is
from online_speculation_b200.arllm.algorithms.mh import (run_mh_chain, run_mh_chains_batched, run_reward_mh_chain,
                                                         suffix_length_probabilities)
from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import ConditionalISConfig, MHConfig, RewardMHConfig, SamplingConfig
from online_speculation_b200.shared.metrics import empirical_distribution, total_variation
from online_speculation_b200.shared.rng import SeedStream


def _small_backend():
    # a genuinely prefix-dependent 3-token model
    def row(prefix):
        h = (sum(prefix) * 7 + len(prefix) * 3) % 5
        base = np.array([1.0 + h, 2.0, 0.5 + 0.5 * h])
        return base / base.sum()
    return TabularBackend(row, 3)


def _power_target(backend, prompt, L, alpha):
    probs = {}
    for seq in itertools.product(range(3), repeat=L):
        lp = sum(backend.score_batch_one(prompt, seq)) if hasattr(backend, "score_batch_one") else None
        ctx = list(prompt)
        logp = 0.0
        for t in seq:
            logp += math.log(backend.probabilities(tuple(ctx))[t])
            ctx.append(t)
        probs[seq] = math.exp(alpha * logp)
    z = sum(probs.values())
    return {k: v / z for k, v in probs.items()}


def test_seed_stream_matches_reference_golden():
    assert SeedStream(7).derive("mh", 0, 1, "cut") == 2192523971420706700
    assert SeedStream(2**100 + 5).derive(None, True, 1.5, b"x", "é") == 5596754170960564003


def test_suffix_schedules_have_full_support():
    for schedule in ("uniform", "inverse_length", "multiscale"):
        p = suffix_length_probabilities(10, schedule)
        assert abs(sum(p) - 1) < 1e-12 and min(p) > 0


def test_power_mh_matches_enumerated_target():
    backend = _small_backend()
    prompt = (1,)
    L, alpha = 3, 2.0
    target = _power_target(backend, prompt, L, alpha)
    cfg = MHConfig(alpha=alpha, total_length=L, block_size=L, iterations=6)
    chains = run_mh_chains_batched(backend, prompt, cfg, SamplingConfig(temperature=1 / alpha),
                                   [SeedStream(s) for s in range(3000)], chain_ids=list(range(3000)))
    emp = empirical_distribution(c.token_ids for c in chains)
    assert total_variation(emp, target) < 0.05


def test_batched_chains_equal_sequential():
    backend = _small_backend()
    cfg = MHConfig(alpha=3.0, total_length=4, block_size=2, steps_per_block=2)
    prop = SamplingConfig(temperature=1 / 3)
    seeds = [SeedStream(11), SeedStream(12)]
    batched = run_mh_chains_batched(backend, (0,), cfg, prop, seeds, chain_ids=[4, 9])
    single = [run_mh_chain(backend, (0,), cfg, prop, s, chain_id=c) for s, c in zip(seeds, [4, 9])]
    for a, b in zip(batched, single):
        assert a.token_ids == b.token_ids and a.trace == b.trace


def _toy_oracle(backend, L, tau):
    """Per-position marginals of pi_r for reward = fraction of zeros: p_t(v) exp([v=0] / (L tau))."""
    p = backend.position_probabilities.copy()
    tilt = np.ones_like(p)
    tilt[:, 0] = math.exp(1.0 / (L * tau))
    m = p * tilt
    return m / m.sum(-1, keepdims=True)


def test_reward_mh_on_positional_toy_matches_factorised_oracle():
    V, L, tau = 32, 12, 0.5
    backend = TabularBackend.per_position_logits(V, L, seed=3, prompt_length=2)
    reward = lambda prompt, y: sum(t == 0 for t in y) / len(y)
    cfg = RewardMHConfig(total_length=L, block_size=L, reward_temperature=tau, iterations=64)
    chains = [run_reward_mh_chain(backend, (5, 6), cfg, SamplingConfig(), reward, SeedStream(s), chain_id=0)
              for s in range(400)]
    oracle = _toy_oracle(backend, L, tau)
    zeros = np.array([[c.token_ids[t] == 0 for t in range(L)] for c in chains], dtype=np.float64)
    emp = zeros.mean(0)
    # standard error ~ sqrt(p(1-p)/400) <= 0.025
    assert np.all(np.abs(emp - oracle[:, 0]) < 0.08)
    # expected count of zeros (exact Poisson-binomial mean)
    assert abs(zeros.sum(1).mean() - oracle[:, 0].sum()) < 0.25


def test_conditional_is_on_positional_toy():
    V, L, tau = 32, 12, 0.5
    backend = TabularBackend.per_position_logits(V, L, seed=5, prompt_length=1)
    reward = lambda prompt, y: sum(t == 0 for t in y) / len(y)
    cfg = ConditionalISConfig(candidate_count=8, rollout_count=4, block_size=4, total_length=L,
                              reward_temperature=tau)
    runs = [run_conditional_is(base_backend=backend, prompt=(9,), config=cfg, seeds=SeedStream(s), reward=reward)
            for s in range(150)]
    oracle = _toy_oracle(backend, L, tau)
    zeros = np.array([[r.token_ids[t] == 0 for t in range(L)] for r in runs], dtype=np.float64)
    # finite-candidate SIR is approximately exact; the tilt towards zeros must show up
    assert zeros.sum(1).mean() > backend.position_probabilities[:, 0].sum() - 0.2
    assert abs(zeros.sum(1).mean() - oracle[:, 0].sum()) < 0.4
    assert all(len(r.steps) == 3 for r in runs)


def test_off_policy_conditional_is_uses_importance_ratio():
    V, L = 8, 4
    backend = TabularBackend.per_position_logits(V, L, seed=9, prompt_length=1)
    cfg = ConditionalISConfig(candidate_count=2, rollout_count=2, block_size=2, total_length=L, reward_temperature=1)
    res = run_conditional_is(base_backend=backend, prompt=(1,), config=cfg, seeds=SeedStream(0),
                             reward=lambda p, y: 0.0, rollout_sampling=SamplingConfig(temperature=2.0))
    ev = res.steps[0].candidates[0].rollouts[0]
    assert ev.raw_log_importance_ratio == pytest.approx(ev.base_logprob - ev.proposal_logprob)


def _exact_conditional_is_law(p, reward, tau):
    """Exact law of conditional IS with 2 candidates and 1 rollout on a 2-token model.

    Step 1: candidates c1, c2 ~ p[0]; each gets one rollout y ~ p[1] and weight exp(r(c, y) / tau);
    c_k is kept with probability w_k / (w_1 + w_2).  Step 2 (the last block, no rollout): candidates
    d1, d2 ~ p[1] with weights exp(r(a, d) / tau).  Returns P(a, b) for every (a, b).
    """
    V = p.shape[1]
    first = np.zeros(V)
    for c1, c2, y1, y2 in itertools.product(range(V), repeat=4):
        w1, w2 = math.exp(reward((c1, y1)) / tau), math.exp(reward((c2, y2)) / tau)
        pr = p[0, c1] * p[0, c2] * p[1, y1] * p[1, y2]
        first[c1] += pr * w1 / (w1 + w2)
        first[c2] += pr * w2 / (w1 + w2)
    law = {}
    for a in range(V):
        second = np.zeros(V)
        for d1, d2 in itertools.product(range(V), repeat=2):
            w1, w2 = math.exp(reward((a, d1)) / tau), math.exp(reward((a, d2)) / tau)
            pr = p[1, d1] * p[1, d2]
            second[d1] += pr * w1 / (w1 + w2)
            second[d2] += pr * w2 / (w1 + w2)
        for b in range(V):
            law[(a, b)] = first[a] * second[b]
    return law


def test_conditional_is_matches_its_exact_finite_candidate_law():
    """Not the tilted target (finite K and R bias it) but the sampler's own exact law, enumerated."""
    V, L, tau = 3, 2, 0.5
    backend = TabularBackend.per_position_logits(V, L, seed=21, prompt_length=1)

    def reward(y):
        return float(y[0] == 0) + 0.5 * float(y[1] == y[0])

    law = _exact_conditional_is_law(backend.position_probabilities, reward, tau)
    assert abs(sum(law.values()) - 1) < 1e-12
    cfg = ConditionalISConfig(candidate_count=2, rollout_count=1, block_size=1, total_length=L, reward_temperature=tau)
    runs = [run_conditional_is(base_backend=backend, prompt=(2,), config=cfg, seeds=SeedStream(1000 + s),
                               reward=lambda prompt, y: reward(y))
            for s in range(4000)]
    emp = empirical_distribution(tuple(r.token_ids) for r in runs)
    # 9 outcomes, 4000 runs: sampling noise alone gives a TV of about 0.02
    assert total_variation(emp, law) < 0.045
