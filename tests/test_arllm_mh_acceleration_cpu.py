"""Exactness tests of the reward-MH accelerations on tabular models (CPU)."""

import math

import numpy as np
import pytest

from online_speculation_b200.arllm.algorithms.mh import run_reward_mh_chain
from online_speculation_b200.arllm.algorithms.mh_acceleration import (FrozenReplaySuffixProposal,
                                                                      run_reward_mh_chain_delayed,
                                                                      run_reward_mh_chain_prefetched,
                                                                      run_reward_mh_chain_replay_proposal,
                                                                      run_reward_mh_chains_replay_proposal)
from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import RewardMHConfig, SamplingConfig
from online_speculation_b200.arllm.types import ScoreRequest
from online_speculation_b200.shared.rng import SeedStream


def _zeros(prompt, y):
    return sum(t == 0 for t in y) / len(y)


def _oracle(backend, L, tau):
    p = backend.position_probabilities.copy()
    p[:, 0] *= math.exp(1.0 / (L * tau))
    return p / p.sum(-1, keepdims=True)


@pytest.mark.parametrize("proposal", [SamplingConfig(), SamplingConfig(temperature=1.7)])
def test_prefetched_chain_is_the_plain_chain(proposal):
    backend = TabularBackend.per_position_logits(12, 8, seed=4, prompt_length=1)
    cfg = RewardMHConfig(total_length=8, block_size=8, reward_temperature=0.3, iterations=20)
    for s in range(5):
        plain = run_reward_mh_chain(backend, (3,), cfg, proposal, _zeros, SeedStream(s), chain_id=2)
        fast = run_reward_mh_chain_prefetched(backend, (3,), cfg, proposal, _zeros, SeedStream(s), chain_id=2)
        assert fast.chain.token_ids == plain.token_ids
        assert fast.chain.trace == plain.trace
        assert fast.chain.reward == plain.reward
        snap = fast.prefetch
        assert snap.used_proposals == 20 and snap.reward_evaluations == 21
        assert snap.prefetched_proposals == 1 + 2 * 19
        assert snap.unused_prefetched_proposals == snap.prefetched_proposals - 20


def test_delayed_acceptance_targets_the_tilted_model():
    V, L, tau = 16, 6, 0.4
    backend = TabularBackend.per_position_logits(V, L, seed=11, prompt_length=1)
    cfg = RewardMHConfig(total_length=L, block_size=L, reward_temperature=tau, iterations=40)
    surrogate = lambda p, y: 0.5 * _zeros(p, y) + 0.05 * (y[0] % 3)   # deliberately biased surrogate
    runs = [run_reward_mh_chain_delayed(backend, (7,), cfg, SamplingConfig(), _zeros, surrogate, SeedStream(s))
            for s in range(400)]
    emp = np.array([[r.token_ids[t] == 0 for t in range(L)] for r in runs], dtype=np.float64).mean(0)
    assert np.all(np.abs(emp - _oracle(backend, L, tau)[:, 0]) < 0.09)
    r = runs[0]
    assert r.surrogate_reward_evaluations == 41
    assert r.exact_reward_evaluations == 1 + sum(s.stage_one_accepted for s in r.trace)
    for s in r.trace:
        assert s.accepted <= s.stage_one_accepted
        assert (s.proposed_reward is None) == (not s.exact_reward_evaluated)


def test_delayed_acceptance_with_exact_surrogate_never_rejects_in_stage_two():
    backend = TabularBackend.per_position_logits(10, 5, seed=2, prompt_length=1)
    cfg = RewardMHConfig(total_length=5, block_size=5, reward_temperature=0.5, iterations=30)
    r = run_reward_mh_chain_delayed(backend, (1,), cfg, SamplingConfig(), _zeros, _zeros, SeedStream(3))
    for s in r.trace:
        if s.stage_one_accepted:
            assert s.stage_two_log_acceptance == pytest.approx(0.0) and s.accepted


def test_replay_proposal_mixture_probabilities_are_exact():
    backend = TabularBackend.per_position_logits(6, 3, seed=1, prompt_length=1)
    prop = FrozenReplaySuffixProposal(backend, history_mixture=0.4)
    prop.observe_sequences((2,), [(0, 1, 2), (0, 1, 2), (3, 1, 2)])
    with pytest.raises(RuntimeError):
        prop.draw((2,), 3, seed=0, request_id="x")
    prop.freeze()
    with pytest.raises(RuntimeError):
        prop.observe_suffix((2,), (1,))
    base = sum(backend.score_batch([ScoreRequest((2,), ((0, 1, 2),), None)])[0])
    want = math.log(0.6 * math.exp(base) + 0.4 * (2 / 3))
    assert prop.logprob((2,), (0, 1, 2)) == pytest.approx(want, rel=1e-9)
    # a suffix never observed keeps only the base component
    lp = prop.logprob((2,), (5, 5, 5), base_logprob=-3.0)
    assert lp == pytest.approx(math.log(0.6) - 3.0)
    # a prefix with no history is the base proposal itself
    assert prop.logprob((2, 5), (1, 2), base_logprob=-1.5) == pytest.approx(-1.5)
    draws = [prop.draw((2,), 3, seed=s, request_id=f"d{s}") for s in range(200)]
    frac = np.mean([d.source == "history" for d in draws])
    assert abs(frac - 0.4) < 0.1
    for d in draws[:20]:
        assert d.proposal_logprob == pytest.approx(prop.logprob((2,), d.token_ids,
                                                                base_logprob=sum(d.base_token_logprobs)))
    snap = prop.snapshot()
    assert snap.stored_suffixes == 9 and snap.history_draws + snap.base_draws == 200


def test_replay_proposal_chain_targets_the_tilted_model():
    V, L, tau = 8, 5, 0.5
    backend = TabularBackend.per_position_logits(V, L, seed=6, prompt_length=1)
    prop = FrozenReplaySuffixProposal(backend, history_mixture=0.3)
    rng = np.random.default_rng(0)
    # a deliberately skewed history: many all-zero suffixes
    prop.observe_sequences((4,), [tuple(int(x) for x in rng.integers(0, 2, size=L)) for _ in range(30)])
    cfg = RewardMHConfig(total_length=L, block_size=L, reward_temperature=tau, iterations=30)
    runs = run_reward_mh_chains_replay_proposal(prop, (4,), cfg, _zeros, SeedStream(9), chains=300)
    emp = np.array([[r.token_ids[t] == 0 for t in range(L)] for r in runs], dtype=np.float64).mean(0)
    assert np.all(np.abs(emp - _oracle(backend, L, tau)[:, 0]) < 0.1)
    assert any(s.proposal_source == "history" for r in runs for s in r.trace)
    one = run_reward_mh_chain_replay_proposal(prop, (4,), cfg, _zeros, SeedStream(9), chain_id=0)
    assert one.token_ids == runs[0].token_ids
