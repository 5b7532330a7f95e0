"""Rollout broker, replay store lifecycle, base replay, token tree and streaming rewards on the tabular backend."""

import numpy as np
import pytest

from online_speculation_b200.arllm.acceleration import (ActiveBatchSpeculationConfig, LowPriorityRunAheadBackend,
                                                        RolloutTokenTree, StreamingRewardEvaluator)
from online_speculation_b200.arllm.algorithms.base_replay import run_base_replay
from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.config import BaseReplayConfig, SamplingConfig
from online_speculation_b200.arllm.replay import (BehaviorPolicy, BehaviorRegistry, InMemoryReplayStore, ReplayKey,
                                                  ReplaySampleRequest, mixture_logprobabilities,
                                                  sample_replay_records, validate_record_probabilities)
from online_speculation_b200.arllm.rollout_broker import AsyncRolloutBroker, PartialRollout
from online_speculation_b200.arllm.types import GenerationRequest, ScoreRequest
from online_speculation_b200.shared.rng import SeedStream

V = 6


def _tab(seed=0, name="tab"):
    rng = np.random.default_rng(seed)
    t = {}

    def row(prefix):
        k = tuple(prefix[-1:])
        if k not in t:
            t[k] = rng.dirichlet(np.ones(V))
        return t[k]
    return TabularBackend(row, V, model_id=name)


def reward(prompt, comp):
    return float(sum(1 for x in comp if x == 0))


def test_broker_resumes_partial_rollouts_exactly():
    b = _tab()
    reqs = [GenerationRequest((1,), 10, SamplingConfig(), seed=s, request_id=f"r{s}") for s in range(5)]
    res = AsyncRolloutBroker(b, chunk_tokens=3, max_batch_size=2).run_until(reqs, completion_target=2)
    assert len(res.completed) >= 2 and res.snapshot.partial_rollouts == 5 - len(res.completed)
    rest = AsyncRolloutBroker(b, chunk_tokens=4).run_until(res.partial)
    allc = {s.request_id: s for s in res.completed + rest.completed}
    assert len(allc) == 5
    for s in allc.values():
        assert len(s.token_ids) == 10
        sc = b.score_batch([ScoreRequest(s.prefix, (s.token_ids,), None)])[0]
        assert sc == pytest.approx(s.token_logprobs)
    with pytest.raises(ValueError):
        PartialRollout(reqs[0], token_ids=(1,), token_logprobs=())


def test_replay_store_claims_are_single_use():
    b = _tab()
    pol = BehaviorPolicy.for_backend(b, SamplingConfig(temperature=1.5), label="hot")
    reg = BehaviorRegistry([pol])
    key = ReplayKey((1,), (), (2,), "v1")
    recs = sample_replay_records(pol, [ReplaySampleRequest(key, 4, s, f"id{s}") for s in range(3)], reward)
    store = InMemoryReplayStore()
    for r in recs:
        store.add_evaluation(r)
    assert store.inventory(key) == {"hot": 3}
    (claim,) = store.freeze_claims([key], 2)
    assert claim.count == 2 and store.evaluation_count == 1
    got = store.reveal_and_consume(claim)
    assert len(got) == 2 and store.design_count == 2
    with pytest.raises(ValueError):
        store.reveal_and_consume(claim)
    validate_record_probabilities(got, reg)
    mix = mixture_logprobabilities(reg, key, {"hot": 2}, [r.completion for r in got])
    assert mix == pytest.approx([r.behavior_logprob for r in got])


def test_base_replay_runs_with_reserve_history():
    b = _tab(1)
    reserve = BehaviorPolicy.for_backend(_tab(1, "tab"), SamplingConfig(temperature=1.3), label="reserve")
    res = run_base_replay(b, BehaviorRegistry(), InMemoryReplayStore(), (1,),
                          BaseReplayConfig(candidate_count=3, block_size=2, total_length=6, fresh_rollouts=2,
                                           reserve_rollouts=4, max_history_per_candidate=3),
                          SamplingConfig(), reward, SeedStream(0), reserve_policy=reserve)
    assert len(res.token_ids) == 6 and res.reserve_records_written > 0
    for st in res.steps:
        assert abs(sum(np.exp(c.estimate.log_weight) for c in st.candidates)) > 0


def test_token_tree_drafts_and_run_ahead():
    tree = RolloutTokenTree(max_context_tokens=3, min_context_tokens=2, min_token_probability=0.3)
    for _ in range(3):
        tree.observe((1, 2, 3, 4, 5))
    d = tree.draft((9, 1, 2), 3)
    assert d.token_ids == (3, 4, 5) and d.matched_context_tokens == 2
    tree.record_verification(proposed=3, accepted=2)
    assert tree.snapshot().acceptance_rate == pytest.approx(2 / 3)
    cfg = ActiveBatchSpeculationConfig()
    assert cfg.draft_tokens(3) == 8 and cfg.draft_tokens(10) == 4 and cfg.draft_tokens(600) == 0
    b = _tab()
    t2 = RolloutTokenTree()
    with LowPriorityRunAheadBackend(b, t2, chunk_tokens=4) as ra:
        ra.submit_run_ahead([GenerationRequest((1,), 10, SamplingConfig(), 5, "bg")])
        ra.wait_for_run_ahead()
        out = ra.sample_batch([GenerationRequest((2,), 3, SamplingConfig(), 1, "fg")])
        assert len(out[0].token_ids) == 3
        assert ra.snapshot().completed_tokens >= 10 and t2.snapshot().observed_sequences >= 1


def test_streaming_rewards_match_direct_evaluation():
    b = _tab()
    reqs = [GenerationRequest((1,), 5, SamplingConfig(), s, f"s{s}") for s in range(4)]
    with StreamingRewardEvaluator(workers=2) as ev:
        samples, rewards, snap = ev.sample_and_score(b, reqs, [((1,), ())] * 4, reward)
    assert rewards == tuple(reward((1,), s.token_ids) for s in samples) and snap.submitted_rewards == 4


def test_declared_logprob_tolerance_is_found_through_wrappers():
    from online_speculation_b200.arllm.backends.batching import ContinuousBatchingBackend
    from online_speculation_b200.arllm.backends.cache import ScoreCachingBackend
    from online_speculation_b200.arllm.replay import declared_logprob_tolerance

    inner = _tab(1)
    assert declared_logprob_tolerance(inner) is None
    inner.logprob_tolerance = (1e-3, 2e-2)
    wrapped = ScoreCachingBackend(ContinuousBatchingBackend(inner))
    try:
        assert declared_logprob_tolerance(wrapped) == (1e-3, 2e-2)
    finally:
        wrapped._backend.close()


def test_chunked_resumed_rollouts_follow_the_policy_law():
    """Rollouts advanced one token per segment (fresh seed per segment) have the policy's exact law."""
    import itertools
    import math

    from online_speculation_b200.shared.metrics import empirical_distribution, total_variation

    b = _tab(3)
    pol = SamplingConfig(temperature=0.8)
    law = {}
    for seq in itertools.product(range(b.vocab_size), repeat=3):
        ctx, lp = [2], 0.0
        for t in seq:
            lp += math.log(b.probabilities(tuple(ctx), pol)[t])
            ctx.append(t)
        law[seq] = math.exp(lp)
    reqs = [GenerationRequest((2,), 3, pol, seed=s, request_id=f"c{s}") for s in range(12000)]
    res = AsyncRolloutBroker(b, chunk_tokens=1, max_batch_size=1024).run_until(reqs)
    assert len(res.completed) == 12000 and all(len(s.token_ids) == 3 for s in res.completed)
    emp = empirical_distribution(tuple(s.token_ids) for s in res.completed)
    # 216 outcomes, 12000 draws: exact samples alone show a TV of 0.033 (at most 0.04 in 20 trials)
    assert total_variation(emp, law) < 0.055
