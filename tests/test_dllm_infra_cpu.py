"""CPU test of the dLLM infrastructure families on the block-diffusion backend over a tiny module
(arm layout, equal work per arm, reuse and evaluation counters)."""

import torch

from online_speculation_b200.dllm import DiffusionEngineBackend, DiffusionSamplingConfig, ModuleLogits
from online_speculation_b200.experiments.dllm_infra import FAMILIES, run_families


class _Tiny(torch.nn.Module):
    def __init__(self, V=13, H=16):
        super().__init__()
        self.emb = torch.nn.Embedding(V, H)
        self.mix = torch.nn.Linear(H, H)
        self.out = torch.nn.Linear(H, V)

    def forward(self, t):
        x = self.emb(t)
        return self.out(x + torch.tanh(self.mix(x.mean(1, keepdim=True))))


def test_every_family_runs_both_arms():
    torch.manual_seed(0)
    be = DiffusionEngineBackend(ModuleLogits(_Tiny(), mask_token_id=12), model_id="tiny")
    sp = DiffusionSamplingConfig(block_length=2, steps_per_block=2, temperature=1.0, remasking="random",
                                 mask_token_id=12)
    rep = run_families(be, prompt=(1, 2, 3), sampling=sp, block=2, generation=4, reward_delay=0.0)
    assert list(rep) == list(FAMILIES)
    b = rep["block_continuous_batching"]
    assert b["sequential"]["tokens"] == b["batched"]["tokens"] == 8
    r = rep["resume_committed_blocks"]
    assert r["restart_after_interruption"]["tokens"] == r["resume_committed"]["tokens"] == 4
    s = rep["streaming_reward"]
    assert s["after_batch"]["rewards"] == s["thread_pool"]["rewards"]      # same draws, same rewards
    m = rep["delayed_acceptance_mh"]
    assert m["delayed_acceptance"]["exact_reward_evaluations"] <= m["reward_mh"]["exact_reward_evaluations"]
    assert rep["block_smc_rollout_forest"]["no_reuse"]["reused_rollouts"] == 0
    assert rep["block_smc_rollout_forest"]["reuse"]["reused_rollouts"] > 0
    assert all(v["telemetry"]["wall_seconds"] >= 0 for arms in rep.values() for v in arms.values())
