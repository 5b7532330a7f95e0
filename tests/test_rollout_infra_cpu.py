"""CPU test of the rollout-infrastructure benchmark harness on the exact tabular backend
(arms, record layout, agreement metric); the engine arms run in the GPU suite."""

import numpy as np

from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.experiments.rollout_infra import agreement, run_benchmark


def test_harness_runs_every_arm_on_the_tabular_backend():
    made = []

    def make(spec):
        made.append(spec)
        return TabularBackend.per_position_logits(16, 12, seed=2, prompt_length=3)

    rep = run_benchmark(make, prompts=[(1, 2, 3), (4, 5, 6)], max_new_tokens=8, batch_sizes=(2, 1),
                        history_rollouts=1, draft_tokens=4, block_size=4, candidates=2, rollouts=2, mh_updates=6,
                        verifier_delay=0.0)
    assert [a["name"] for a in rep["decode"]] == ["plain", "rollout_tree"]
    assert [a["name"] for a in rep["algorithm"]] == ["conditional_plain", "conditional_rollout_tree",
                                                     "smc_no_reuse", "smc_reuse"]
    assert made[0] is None and made[1] is not None and made[1].draft_tokens(2) == 4
    plain, tree = rep["decode"]
    assert plain["online"]["sequences"] == 2 * (2 + 1) and plain["online"]["output_tokens"] == 48
    assert tree["cache_build"]["sequences"] == 2 and plain["cache_build"]["sequences"] == 0
    # the same seeds on the same exact backend: identical draws
    assert tree["online"]["agreement_with_plain"] == {"identical_requests": 1.0, "mean_matching_prefix": 1.0}
    smc = rep["algorithm"][3]["online"]["diagnostics"]
    assert len(smc) == 2 and all("reused_rollouts" in d for d in smc)
    assert all(np.isfinite(a["online"]["output_tokens_per_second"]) for a in rep["algorithm"])
    reuse = {a["name"]: a["online"] for a in rep["reuse"]}
    assert set(reuse) == {"mh_standard", "mh_prefetched", "mh_delayed"}
    # prefetching changes when proposals are generated, not which: the same chain
    assert reuse["mh_prefetched"]["identical_to_standard"]
    assert reuse["mh_delayed"]["exact_reward_evaluations"] <= reuse["mh_standard"]["exact_reward_evaluations"]


def test_agreement_metric():
    base = {"a": (1, 2, 3, 4), "b": (5, 6)}
    assert agreement(base, base) == {"identical_requests": 1.0, "mean_matching_prefix": 1.0}
    got = agreement({"a": (1, 2, 9, 9), "b": (5, 6)}, base)
    assert got["identical_requests"] == 0.5 and got["mean_matching_prefix"] == (0.5 + 1.0) / 2
