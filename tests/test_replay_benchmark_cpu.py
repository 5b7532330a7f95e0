"""CPU test of the replay benchmarks (base replay fresh vs warm; dynamic IS arms) on the exact
tabular backend: arm layout, reuse counters and output lengths."""

from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.experiments.replay_benchmark import run_benchmark


def test_replay_and_dynamic_is_arms():
    backend = TabularBackend.per_position_logits(16, 12, seed=2, prompt_length=3)

    def reward(_p, y):
        return sum(t == 0 for t in y) / max(1, len(y))

    rep = run_benchmark(backend, prompts=[(1, 2, 3), (4, 5, 6)], length=8, block=4, candidates=3, reward=reward)
    fresh, warm = (a["online"] for a in rep["replay"])
    assert [a["name"] for a in rep["replay"]] == ["fresh_only", "warm_replay"]
    assert fresh["history_rollouts_reused"] == 0 and rep["replay"][0]["cache_build"]["records"] == 0
    # history for every candidate of the first decision (the last one has no rollout left): 2 prompts x 3 x 4
    assert rep["replay"][1]["cache_build"]["records"] == 2 * 3 * 4
    assert warm["history_rollouts_reused"] == 2 * 3 * 4
    assert fresh["output_tokens"] == warm["output_tokens"] == 2 * 8
    assert fresh["decisions"] == warm["decisions"] == 2 * 2
    arms = {a["name"]: a["online"] for a in rep["dynamic_is"]}
    assert list(arms) == ["base_candidate_fixed", "replay_aware_fixed", "replay_aware_optimal"]
    assert arms["base_candidate_fixed"]["auxiliary_candidates"] == 0
    assert arms["base_candidate_fixed"]["history_rollouts_reused"] == 0
    assert all(a["output_tokens"] == 16 and a["mean_candidate_ess"] > 0 for a in arms.values())
    # the prepared store is spent: the allocation reuses history in the replay-aware arms
    assert arms["replay_aware_fixed"]["history_rollouts_reused"] > 0
    assert rep["dynamic_is"][1]["cache_build"]["records"] > 0
    assert 0.0 <= arms["replay_aware_optimal"]["mean_output_reward"] <= 1.0


def test_dynamic_is_arms_run_through_the_method_runner():
    from online_speculation_b200.experiments.methods import MethodSettings, RUNNABLE_AR_METHODS, run_ar_method

    backend = TabularBackend.per_position_logits(16, 12, seed=2, prompt_length=3)
    s = MethodSettings(max_new_tokens=8, block_size=4, candidates=3, rollouts=2)
    for arm in ("base_candidate_fixed", "replay_aware_fixed", "replay_aware_optimal"):
        assert arm in RUNNABLE_AR_METHODS
        out = run_ar_method(arm, backend, (1, 2, 3), s, 7, reward=lambda p, y: sum(t == 0 for t in y) / len(y))
        assert len(out.token_ids) == 8 and out.diagnostics["steps"] == 2
        assert (out.diagnostics["history_rollouts_reused"] > 0) == (arm != "base_candidate_fixed")
