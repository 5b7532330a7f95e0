"""VRPO on CPU: mask plans, the ELBO estimator, shared (antithetic) plans, the loss at initialisation,
LoRA gradients through the MoE model, trainer checkpoints, preference pairs."""

import math

import numpy as np
import pytest
import torch

from online_speculation_b200.dllm.config import VRPOSamplingConfig
from online_speculation_b200.dllm.preferences import select_scored_preference_pair
from online_speculation_b200.dllm.vrpo import (estimate_masked_elbo, estimate_vrpo_preference_loss,
                                               sample_vrpo_mask_plan, vrpo_forward_token_slots)
from online_speculation_b200.models.moe import PRESETS, build_weights, random_state_dict
from online_speculation_b200.training.lora import LoRAConfig
from online_speculation_b200.training.vrpo import LoRAMoEPolicy, VRPOTrainer, VRPOTrainingConfig


def test_mask_plan_layout():
    plan = sample_vrpo_mask_plan(10, VRPOSamplingConfig(timestep_samples=4, masks_per_timestep=2),
                                 np.random.default_rng(0))
    assert len(plan.samples) == 8
    for a, b in zip(plan.samples[0::2], plan.samples[1::2]):
        assert a.timestep_index == b.timestep_index and a.mask_count == b.mask_count
    assert all(1 <= s.mask_count <= 10 for s in plan.samples)
    assert vrpo_forward_token_slots(prompt_length=4, chosen_length=5, rejected_length=6,
                                    config=VRPOSamplingConfig())["total"] == 2 * 8 * (8 + 11)


class Tiny(torch.nn.Module):
    def __init__(self, V=11):
        super().__init__()
        self.emb = torch.nn.Embedding(V, 8)
        self.out = torch.nn.Linear(8, V)

    def forward(self, t):
        class O:
            pass
        o = O()
        x = self.emb(t)
        o.logits = self.out(x + x.mean(1, keepdim=True))
        return o


def test_elbo_matches_direct_cross_entropy():
    torch.manual_seed(0)
    m = Tiny()
    plan = sample_vrpo_mask_plan(5, VRPOSamplingConfig(timestep_samples=3), np.random.default_rng(1))
    prompt, ans = (1, 2), (3, 4, 5, 6, 7)
    got = estimate_masked_elbo(m, prompt=prompt, answer=ans, mask_token_id=10, plan=plan)
    terms = []
    for s in plan.samples:
        x = torch.tensor(prompt + ans)
        x[[2 + p for p in s.positions]] = 10
        lp = m(x[None]).logits[0].log_softmax(-1)
        terms.append(sum(lp[2 + p, ans[p]] for p in s.positions) / (s.mask_count / 5))
    assert float(got) == pytest.approx(float(torch.stack(terms).mean()), rel=1e-5)


def _policy(seed=0):
    cfg = PRESETS["tiny-moe"]
    return LoRAMoEPolicy(build_weights(cfg, random_state_dict(cfg, seed=seed), device="cpu"), LoRAConfig(rank=4))


def test_loss_is_log2_at_init_and_grads_reach_adapters():
    pol = _policy()
    from online_speculation_b200.dllm.vrpo import AdapterDisabledReference

    est = estimate_vrpo_preference_loss(pol, AdapterDisabledReference(pol), prompt=(1, 2, 3), chosen=(4, 5, 6, 7),
                                        rejected=(8, 9, 10, 11), mask_token_id=511,
                                        config=VRPOSamplingConfig(timestep_samples=2), beta=0.1)
    assert float(est.loss) == pytest.approx(math.log(2), abs=1e-6)
    assert est.current_chosen_plan is est.reference_chosen_plan       # shared masks
    est.loss.backward()
    g = pol.flat.grad
    assert g is not None and torch.isfinite(g).all() and g.abs().sum() > 0


def test_trainer_checkpoint_resume_and_fingerprint(tmp_path):
    g = torch.Generator().manual_seed(0)
    pairs = [tuple(tuple(torch.randint(0, 500, (n,), generator=g).tolist()) for n in (4, 6, 6)) for _ in range(3)]
    cfg = VRPOTrainingConfig(learning_rate=1e-2, gradient_accumulation_steps=2,
                             sampling=VRPOSamplingConfig(timestep_samples=2))
    a = VRPOTrainer(_policy(), pairs, cfg)
    a.train_step()
    a.save(tmp_path / "ck.pt")
    a.train_step()
    b = VRPOTrainer(_policy(), pairs, cfg)
    b.resume(tmp_path / "ck.pt")
    b.train_step()
    assert torch.allclose(a.policy.flat.detach(), b.policy.flat.detach(), atol=1e-6)
    other = VRPOTrainer(_policy(), pairs, VRPOTrainingConfig(learning_rate=2e-2))
    with pytest.raises(ValueError):
        other.resume(tmp_path / "ck.pt")


def test_preference_pair_selection():
    p = select_scored_preference_pair(candidate_texts=["a", "b", "c"], candidate_rewards=[0.0, 1.0, 0.0])
    assert (p.chosen, p.rejected, p.chosen_source, p.rejected_source) == ("b", "a", "candidate:1", "candidate:0")
    assert select_scored_preference_pair(candidate_texts=["a", "b"], candidate_rewards=[1.0, 1.0]) is None
    q = select_scored_preference_pair(candidate_texts=["a"], candidate_rewards=[0.0], reference_text="gold",
                                      reference_reward=1.0)
    assert q.chosen == "gold" and q.chosen_source == "dataset_reference_completion"
    with pytest.raises(ValueError):
        select_scored_preference_pair(candidate_texts=["a"], candidate_rewards=[float("nan")])
