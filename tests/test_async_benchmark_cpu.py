"""CPU test of the synchronous vs continuously batched benchmark on the exact tabular backend:
both arms run every prompt, the batching wrapper merges calls, and seeded outputs agree."""

from online_speculation_b200.arllm.backends.tabular import TabularBackend
from online_speculation_b200.arllm.rewards import SequenceLogProbabilityReward
from online_speculation_b200.experiments.async_benchmark import run_benchmark
from online_speculation_b200.experiments.methods import MethodSettings


def test_sync_and_async_arms_agree():
    backend = TabularBackend.per_position_logits(16, 12, seed=4, prompt_length=3)
    prompts = [(1, 2, 3), (4, 5, 6), (7, 8, 9), (3, 2, 1)]
    rep = run_benchmark(backend, prompts=prompts, methods=("best_of_n", "conditional_is", "reward_mh"),
                        settings=MethodSettings(max_new_tokens=8, block_size=4, candidates=3, rollouts=2, best_of=3),
                        workers=4, reward_factory=lambda b: SequenceLogProbabilityReward(b, coefficient=0.5))
    assert list(rep["methods"]) == ["best_of_n", "conditional_is", "reward_mh"]
    for name, r in rep["methods"].items():
        assert r["synchronous"]["output_tokens"] == r["asynchronous"]["output_tokens"] == 4 * 8, name
        # the tabular model computes the same law whatever the batch: seeded draws are identical
        assert r["asynchronous"]["agreement_with_synchronous"]["identical_requests"] == 1.0, name
        assert r["asynchronous"]["batching"], name
