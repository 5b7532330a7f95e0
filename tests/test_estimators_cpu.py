"""CPU tests of the estimator helpers: importance weights, truncated replay, SMC resampling,
self-consistency, FLOP accounting, the GSM8K helpers and the distribution audit.

Each estimator is checked against an exact enumeration where one exists (the truncated
replay estimator's expectation, systematic resampling's count bounds); the reference covers
the same helpers in tests/test_replay.py, tests/test_smc_forest.py, tests/test_gsm8k.py,
tests/test_compute_accounting.py and tests/test_distribution_audit.py.
"""

from __future__ import annotations

import math
from fractions import Fraction

import numpy as np
import pytest

from online_speculation_b200.shared.importance import (MonteCarloRolloutWeightProvider, ProbabilityObservation,
                                                       RolloutObservation, TruncatedReplayRolloutWeightProvider,
                                                       corrected_replay_log_weight, logmeanexp)
from online_speculation_b200.shared.smc import (normalize_smc_log_weights, partition_resampled_reservoirs,
                                                systematic_resample)


# ---- importance weights -------------------------------------------------------------------------------------

def test_logmeanexp_matches_direct_and_handles_extremes():
    v = [0.3, -1.2, 2.5, 0.0]
    assert logmeanexp(v) == pytest.approx(math.log(np.mean(np.exp(v))), rel=1e-12)
    assert logmeanexp([1000.0, 1000.0]) == pytest.approx(1000.0)
    assert logmeanexp([-math.inf, -math.inf]) == -math.inf
    with pytest.raises(ValueError):
        logmeanexp([])


@pytest.mark.parametrize("mode", ["importance", "identity", "none"])
def test_monte_carlo_weight_modes(mode):
    obs = [RolloutObservation(0.5, -2.0, -1.0), RolloutObservation(-0.25, -3.0, -3.5)]
    est = MonteCarloRolloutWeightProvider(reward_temperature=0.5, correction=mode).estimate(obs)
    corr = {"importance": [-1.0, 0.5], "identity": [0.0, 0.0], "none": [0.0, 0.0]}[mode]
    expect = [r / 0.5 + c for r, c in zip([0.5, -0.25], corr)]
    assert [w.log_weight for w in est.rollouts] == pytest.approx(expect)
    assert est.log_weight == pytest.approx(logmeanexp(expect))
    if mode == "none":
        assert est.rollouts[0].raw_log_importance_ratio is None
    elif mode == "identity":
        assert est.rollouts[0].applied_log_importance_ratio == 0.0


def test_monte_carlo_weight_clip_and_validation():
    p = MonteCarloRolloutWeightProvider(reward_temperature=1.0, log_ratio_clip=0.5)
    w = p.weight(RolloutObservation(0.0, 0.0, -3.0))
    assert w.raw_log_importance_ratio == pytest.approx(3.0)
    assert w.applied_log_importance_ratio == pytest.approx(0.5)
    assert w.log_weight == pytest.approx(0.5)
    with pytest.raises(ValueError):
        p.weight(RolloutObservation(0.0, None, -3.0))          # importance needs both densities
    with pytest.raises(ValueError):
        MonteCarloRolloutWeightProvider(reward_temperature=1.0, correction="none", log_ratio_clip=1.0)
    with pytest.raises(ValueError):
        MonteCarloRolloutWeightProvider(reward_temperature=0.0)
    with pytest.raises(ValueError):
        RolloutObservation(math.nan)
    with pytest.raises(ValueError):
        MonteCarloRolloutWeightProvider(reward_temperature=1.0).estimate([])


def _replay_case():
    rng = np.random.default_rng(11)
    p = rng.dirichlet(np.ones(6))
    b = rng.dirichlet(np.ones(6))
    b[5] = 0.0                                   # one outcome the behaviour policy never proposes
    b /= b.sum()
    r = rng.normal(size=6)
    return p, b, r


@pytest.mark.parametrize("c", [0.5, 1.0, 2.0])
def test_truncated_replay_is_exactly_unbiased(c):
    """E_b E_p exp(estimate with one history and one fresh draw) = sum_x p(x) exp(r(x) / tau)."""
    p, b, r = _replay_case()
    tau = 0.7
    truth = float(np.sum(p * np.exp(r / tau)))
    expect = 0.0
    for x in range(6):
        if b[x] == 0:
            continue
        hist = ProbabilityObservation(math.log(p[x]), math.log(b[x]), r[x])
        for y in range(6):
            fresh = ProbabilityObservation(math.log(p[y]), math.log(b[y]) if b[y] > 0 else -math.inf, r[y])
            total, _, _ = corrected_replay_log_weight([hist], [fresh], truncation=c, reward_temperature=tau)
            expect += b[x] * p[y] * math.exp(total)
    assert expect == pytest.approx(truth, rel=1e-12)


def test_truncated_replay_terms_and_provider():
    hist = [ProbabilityObservation(-1.0, -2.0, 0.0), ProbabilityObservation(-2.0, -1.0, 1.0)]
    fresh = [ProbabilityObservation(-1.0, -1.0, 0.0), ProbabilityObservation(-0.5, -2.0, 0.0)]
    est = TruncatedReplayRolloutWeightProvider(truncation=2.0, reward_temperature=1.0).estimate(hist, fresh)
    # history: min(log 2, log p/b) + r
    assert est.history_log_terms == pytest.approx((math.log(2.0), -1.0 + 1.0))
    # fresh: log(1 - c b / p); p = b gives no mass (ratio 1 <= c), p/b = e^1.5 > 2 gives log(1 - 2 e^-1.5)
    assert est.fresh_log_terms[0] == -math.inf
    assert est.fresh_log_terms[1] == pytest.approx(math.log1p(-2.0 * math.exp(-1.5)))
    assert est.history_count == 2 and est.fresh_count == 2
    assert 1.0 <= est.history_ess <= 2.0 and est.fresh_ess == pytest.approx(1.0)
    with pytest.raises(ValueError):
        corrected_replay_log_weight(hist, [], truncation=1.0, reward_temperature=1.0)
    with pytest.raises(ValueError):   # a history draw outside the target's support
        corrected_replay_log_weight([ProbabilityObservation(-math.inf, -1.0, 0.0)], fresh, truncation=1.0,
                                    reward_temperature=1.0)


# ---- SMC ----------------------------------------------------------------------------------------------------

def test_normalize_smc_log_weights():
    probs, ess = normalize_smc_log_weights([0.0, math.log(3.0)])
    assert probs == pytest.approx((0.25, 0.75))
    assert ess == pytest.approx(1.0 / (0.25 ** 2 + 0.75 ** 2))
    probs, ess = normalize_smc_log_weights([5.0] * 4)
    assert ess == pytest.approx(4.0)
    for bad in ([], [0.0, math.inf], [math.nan]):
        with pytest.raises(ValueError):
            normalize_smc_log_weights(bad)


@pytest.mark.parametrize("count", [1, 7, 64])
def test_systematic_resample_counts_stay_within_floor_and_ceil(count):
    rng = np.random.default_rng(5)
    p = rng.dirichlet(np.ones(9) * 0.5)
    for _ in range(200):
        idx = systematic_resample(p, count, rng)
        assert len(idx) == count and list(idx) == sorted(idx)
        n = np.bincount(idx, minlength=p.size)
        assert np.all(n >= np.floor(count * p) - 1e-9) and np.all(n <= np.ceil(count * p) + 1e-9)


def test_systematic_resample_is_unbiased():
    rng = np.random.default_rng(9)
    p = np.array([0.1, 0.05, 0.6, 0.25])
    total = np.zeros(4)
    trials = 4000
    for _ in range(trials):
        total += np.bincount(systematic_resample(p, 3, rng), minlength=4)
    assert total / (3 * trials) == pytest.approx(p, abs=0.01)
    with pytest.raises(ValueError):
        systematic_resample([0.0, 0.0], 2, rng)
    with pytest.raises(ValueError):
        systematic_resample([1.0], 0, rng)


def test_partition_resampled_reservoirs_is_disjoint_round_robin():
    reservoirs = [("a0", "a1", "a2", "a3", "a4"), ("b0",), ("c0", "c1")]
    out = partition_resampled_reservoirs(reservoirs, [0, 0, 2, 0])
    assert out == (("a0", "a3"), ("a1", "a4"), ("c0", "c1"), ("a2",))
    with pytest.raises(ValueError):
        partition_resampled_reservoirs(reservoirs, [3])
    with pytest.raises(ValueError):
        partition_resampled_reservoirs(reservoirs, [])


# ---- self-consistency ---------------------------------------------------------------------------------------

def test_modal_answer_and_consensus_index_tie_rules():
    from online_speculation_b200.shared.evaluation.consensus import consensus_index, modal_answer

    assert modal_answer([Fraction(3), Fraction(1), Fraction(3), Fraction(1), None]) == Fraction(1)
    assert modal_answer([None, None]) is None
    texts = ["#### 5", "#### 7", "#### 5", "#### 7", "#### 5"]
    assert consensus_index(texts, [-3.0, -1.0, -2.0, -0.5, -2.0]) == 2
    # nothing parses: the highest log-probability, earliest on ties
    assert consensus_index(["no", "answer", "here"], [-1.0, -0.5, -0.5]) == 1
    with pytest.raises(ValueError):
        consensus_index(["#### 1"], [])


def test_cumulative_consensus_reward_tracks_running_mode():
    from online_speculation_b200.shared.evaluation.consensus import CumulativeConsensusReward

    decode = {(1,): "#### 4", (2,): "#### 9", (3,): "nothing"}
    reward = CumulativeConsensusReward(lambda toks: decode[tuple(toks)])
    assert reward((), [(1,), (2,), (2,)]) == (0.0, 1.0, 1.0)
    assert reward((), [(1,), (1,), (3,)]) == (1.0, 1.0, 0.0)      # 4 now leads 3 to 2
    assert reward.counts == {Fraction(4): 3, Fraction(9): 2}


# ---- accounting and GSM8K helpers ---------------------------------------------------------------------------

def test_flop_accounting():
    from online_speculation_b200.shared.compute import dense_forward_flops, training_step_flops

    assert dense_forward_flops(7_000_000_000, 10) == 140_000_000_000
    assert training_step_flops(100, 10) == 6 * 100 * 10
    assert training_step_flops(100, 10, trainable_fraction=0.0, recompute=True) == 6 * 100 * 10
    with pytest.raises(ValueError):
        dense_forward_flops(-1, 1)


def test_gsm8k_helpers(tmp_path):
    from online_speculation_b200.shared.evaluation import gsm8k

    probs = tuple(gsm8k.GSM8KProblem(i, f"q{i}", f"#### {i}", Fraction(i)) for i in range(20))
    a = gsm8k.select_problems(probs, 5, seed=3)
    assert a == gsm8k.select_problems(probs, 5, seed=3)
    assert [p.index for p in a] == sorted(p.index for p in a) and len(set(a)) == 5
    assert gsm8k.select_problems(probs, None, seed=0) == probs
    with pytest.raises(ValueError):
        gsm8k.select_problems(probs, 21, seed=0)
    assert gsm8k.gsm8k_prompt("What is 2+2?").startswith("What is 2+2?")
    assert gsm8k.accuracy([True, False, True, True]) == 0.75
    with pytest.raises(ValueError):
        gsm8k.accuracy([])
    f = tmp_path / "test.jsonl"
    f.write_text('{"question": "q", "answer": "#### 3"}\n')
    with pytest.raises(ValueError, match="digest"):      # only the pinned file is accepted
        gsm8k.load_gsm8k(f, download=False)


# ---- reward configuration -----------------------------------------------------------------------------------

def test_reward_temperature_from_config_precedence():
    from online_speculation_b200.arllm.reward_factory import reward_temperature_from_config

    assert reward_temperature_from_config({"reward": {"temperature": 0.3}}, source="consilience") == 0.3
    assert reward_temperature_from_config({}, source="consilience") == 2.0
    assert reward_temperature_from_config({"conditional_is": {"reward_temperature": 0.4}},
                                          source="sequence_log_probability") == 0.4
    assert reward_temperature_from_config({}, source="sequence_log_probability", default=1.5) == 1.5


def test_model_reward_from_config_sources():
    from online_speculation_b200.arllm.backends.tabular import TabularBackend
    from online_speculation_b200.arllm.reward_factory import model_reward_from_config
    from online_speculation_b200.arllm.rewards import SequenceLogProbabilityReward

    backend = TabularBackend.per_position_logits(8, 4, seed=0, prompt_length=1)
    r = model_reward_from_config(backend, {"conditional_is": {"logprob_reward_scale": 0.5}},
                                 source="sequence_log_probability")
    assert isinstance(r, SequenceLogProbabilityReward)
    with pytest.raises(ValueError):
        model_reward_from_config(backend, {}, source="unknown")
    with pytest.raises(ValueError):
        model_reward_from_config(backend, {"reward": {"consilience": {"scope": "partial"}}}, source="consilience")


# ---- distribution audit -------------------------------------------------------------------------------------

def test_distribution_audit_power_target_small():
    from online_speculation_b200.experiments.distribution_audit import audit_power_mh

    out = audit_power_mh(400, 1)
    assert out["passed"], out
    assert 0.0 <= out["tv"] < 0.2


def test_grpo_compute_estimate():
    from online_speculation_b200.shared.compute import (ADAMW_FLOPS_PER_PARAMETER, estimate_grpo_compute,
                                                        estimate_grpo_compute_from_steps)

    e = estimate_grpo_compute(model_sequence_tokens=1000, generated_completions=10, total_parameters=100,
                              trainable_parameters=100, optimizer_steps=2, reference_scoring=True)
    assert e.rollout_generation_forward_token_slots == 990
    assert e.reference_scoring_forward_token_slots == 1000
    assert e.policy_forward_backward_equivalent_token_slots == 3000      # forward + two gradient passes
    assert e.total_forward_equivalent_token_slots == 4990
    assert e.estimated_dense_model_flops == 2 * 100 * 4990
    assert e.estimated_optimizer_flops == ADAMW_FLOPS_PER_PARAMETER * 100 * 2
    lora = estimate_grpo_compute(model_sequence_tokens=1000, generated_completions=10, total_parameters=100,
                                 trainable_parameters=1, optimizer_steps=1, reference_scoring=False, recompute=True)
    assert lora.policy_forward_backward_equivalent_token_slots == 3000 + 10 and lora.reference_scoring_forward_token_slots == 0
    steps = [{"tokens": 500, "completions": 5}, {"tokens": 500, "completions": 5}]
    two = estimate_grpo_compute_from_steps(steps, total_parameters=100, trainable_parameters=100,
                                           reference_scoring=True, world=2)
    assert two.trainer_observed_prompt_plus_completion_tokens == 2000 and two.optimizer_steps == 2
    assert set(two.as_dict()) >= {"estimated_total_petaflops", "definition", "exclusions"}
    with pytest.raises(ValueError):
        estimate_grpo_compute(model_sequence_tokens=5, generated_completions=6, total_parameters=1,
                              trainable_parameters=1, optimizer_steps=1, reference_scoring=True)
