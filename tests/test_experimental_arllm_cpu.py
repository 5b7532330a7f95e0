"""Experimental autoregressive samplers on tabular models against exact tilted marginals (CPU)."""

import math

import numpy as np
import pytest

from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import (DynamicISConfig, IteratedConditionalISConfig, ProgressiveISConfig,
                                                  SamplingConfig, SMCForestConfig)
from online_speculation_b200.arllm.replay import BehaviorRegistry, InMemoryReplayStore
from online_speculation_b200.experimental.arllm.dynamic_is import (CandidateProposal, empirical_design_statistics,
                                                                    run_dynamic_is)
from online_speculation_b200.experimental.arllm.iterated_is import run_iterated_conditional_is
from online_speculation_b200.experimental.arllm.progressive_is import run_progressive_conditional_is
from online_speculation_b200.experimental.arllm.smc_forest import run_smc_rollout_forest
from online_speculation_b200.experimental.arllm.streaming_is import (FrozenStreamingISEstimator,
                                                                      ordinary_importance_log_weight)
from online_speculation_b200.shared.rng import SeedStream

V, L, TAU = 10, 6, 0.5


def _zeros(prompt, y):
    return sum(t == 0 for t in y) / len(y)


def _backend(seed=7):
    return TabularBackend.per_position_logits(V, L, seed=seed, prompt_length=1)


def _expected_zeros(backend):
    p = backend.position_probabilities[:, 0]
    t = p * math.exp(1 / (L * TAU))
    return float((t / (t + 1 - p)).sum())


def _mean_zeros(runs):
    return float(np.mean([sum(t == 0 for t in r.token_ids) for r in runs]))


def test_iterated_conditional_is_targets_the_tilted_model():
    b = _backend()
    cfg = IteratedConditionalISConfig(pool_size=3, updates=3, rollout_count=3, block_size=2, total_length=L,
                                      reward_temperature=TAU)
    runs = [run_iterated_conditional_is(b, (4,), cfg, _zeros, SeedStream(s)) for s in range(150)]
    assert abs(_mean_zeros(runs) - _expected_zeros(b)) < 0.35
    st = runs[0].steps[0]
    assert len(st.evaluated_candidates) == cfg.fresh_candidate_evaluations
    assert st.candidates[st.selected_index] is st.selected
    assert runs[0].reused_pool_entries == cfg.updates * len(runs[0].steps)


def test_streaming_is_is_order_invariant_and_frozen():
    lw = {("a", 0): 0.3, ("b", 0): -1.0, ("c", 1): 2.0, ("d", 1): 0.1}
    finals = []
    for order in (["a", "b", "c", "d"], ["d", "c", "b", "a"]):
        seen = []
        est = FrozenStreamingISEstimator(2, on_update=lambda snap, c: seen.append(snap.received_fresh))
        est.add_history("h0", 1, 0.5)
        est.freeze([["a", "b"], ["c", "d"]])
        with pytest.raises(RuntimeError):
            est.add_history("h1", 0, 0.0)
        for sid in order:
            k = 0 if sid in "ab" else 1
            est.consume_fresh(sid, k, lw[(sid, k)])
        with pytest.raises(ValueError):
            est.consume_fresh("a", 0, 0.3)
        assert est.complete
        finals.append(est.final_log_weights())
    assert finals[0] == pytest.approx(finals[1])
    est = FrozenStreamingISEstimator(1)
    est.freeze([["x"]])
    with pytest.raises(ValueError):
        est.consume_fresh("y", 0, 0.0)
    with pytest.raises(RuntimeError):
        est.final_log_weights()
    assert ordinary_importance_log_weight(reward=1.0, reward_temperature=0.5, target_logprob=-1.0,
                                          behavior_logprob=-2.0) == pytest.approx(3.0)


def test_smc_forest_targets_the_tilted_model_and_reuses_rollouts():
    b = _backend(3)
    cfg = SMCForestConfig(particle_count=8, branch_factor=2, rollout_count=3, block_size=2, total_length=L,
                          reward_temperature=TAU, reward_workers=2)
    runs = [run_smc_rollout_forest(b, (4,), cfg, _zeros, SeedStream(s)) for s in range(100)]
    assert abs(_mean_zeros(runs) - _expected_zeros(b)) < 0.4
    assert sum(r.reused_rollouts for r in runs) > 0
    batch = run_smc_rollout_forest(b, (4,), cfg, None, SeedStream(1),
                                   reward_batch=lambda p, ys: [_zeros(p, y) for y in ys])
    assert len(batch.token_ids) == L


def test_progressive_is_allocates_independent_evaluations():
    b = _backend(5)
    cfg = ProgressiveISConfig(candidate_count=4, pilot_rollouts_per_candidate=2, evaluation_cost_budget=12.0,
                              block_size=2, total_length=L, reward_temperature=TAU, reward_workers=2)
    runs = [run_progressive_conditional_is(b, (4,), cfg, _zeros, SeedStream(s)) for s in range(100)]
    assert abs(_mean_zeros(runs) - _expected_zeros(b)) < 0.4
    st = runs[0].steps[0]
    assert all(c.evaluation_count >= 1 for c in st.candidates)
    assert all(len(c.evaluation_rollouts) == c.evaluation_count for c in st.candidates)
    assert st.frozen_evaluation_cost > 0


def test_dynamic_is_with_a_defensive_auxiliary_mixture():
    b = _backend(9)
    hot = CandidateProposal.for_backend(b, SamplingConfig(temperature=2.0), label="hot")
    cfg = DynamicISConfig(candidate_count=4, block_size=2, total_length=L, reward_temperature=TAU,
                          max_history_per_candidate=4, truncation=8.0, reserve_rollouts=2, rollout_budget=12.0,
                          auxiliary_mixture=0.3)
    runs = []
    for s in range(80):
        reg, store = BehaviorRegistry(), InMemoryReplayStore()
        runs.append(run_dynamic_is(b, reg, store, (4,), cfg, _zeros, "v1", SeedStream(s), auxiliary_proposal=hot,
                                   statistics_provider=empirical_design_statistics))
    assert abs(_mean_zeros(runs) - _expected_zeros(b)) < 0.45
    draws = [c.draw for r in runs for st in r.steps for c in st.candidates]
    assert any(d.source == "auxiliary" for d in draws) and any(d.source == "base" for d in draws)
    for d in draws[:20]:
        want = np.logaddexp(math.log(0.7) + d.base_logprob, math.log(0.3) + d.auxiliary_logprob)
        assert d.proposal_logprob == pytest.approx(want)
    assert sum(r.reserve_records_written for r in runs) > 0
    with pytest.raises(ValueError):
        run_dynamic_is(b, BehaviorRegistry(), InMemoryReplayStore(), (4,), cfg, _zeros, "v1", SeedStream(0))


def _context_model(seed, V=4):
    rng = np.random.default_rng(seed)
    table = {}

    def row(prefix):
        k = tuple(prefix[-2:])
        if k not in table:
            table[k] = rng.dirichlet(np.ones(V) * 0.7)
        return table[k]
    return TabularBackend(row, V, model_id=f"ctx{seed}")


@pytest.mark.parametrize("temperature", [1.0, 0.7])
def test_draft_model_speculation_is_exact(temperature):
    import itertools

    from online_speculation_b200.arllm.acceleration import DraftModelSpeculationConfig
    from online_speculation_b200.arllm.types import GenerationRequest
    from online_speculation_b200.experimental.arllm.draft_model_speculation import DraftModelSpeculativeBackend

    target, draft = _context_model(1), _context_model(2)
    spec = DraftModelSpeculativeBackend(target, draft, config=DraftModelSpeculationConfig(draft_tokens=2,
                                                                                           single_request_only=False))
    pol = SamplingConfig(temperature=temperature)
    Lq = 3
    reqs = [GenerationRequest((1,), Lq, pol, seed=s, request_id=f"r{s}") for s in range(6000)]
    out = spec.sample_batch(reqs)
    emp = {}
    for s in out:
        emp[s.token_ids] = emp.get(s.token_ids, 0) + 1
        assert len(s.token_ids) == Lq
    exact = {}
    for seq in itertools.product(range(4), repeat=Lq):
        p = 1.0
        for i in range(Lq):
            p *= target.probabilities((1,) + seq[:i], pol)[seq[i]]
        exact[seq] = p
    tv = 0.5 * sum(abs(emp.get(k, 0) / len(out) - v) for k, v in exact.items())
    assert tv < 0.04
    # returned log-probabilities are the target's
    s = out[0]
    want = [float(np.log(target.probabilities((1,) + s.token_ids[:i], pol)[t])) for i, t in enumerate(s.token_ids)]
    assert s.token_logprobs == pytest.approx(want)
    snap = spec.snapshot()
    assert 0 < snap.draft_tokens_accepted <= snap.draft_tokens_proposed
    assert snap.mean_tokens_per_round > 1.0
