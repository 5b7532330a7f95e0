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
from online_speculation_b200.training.vrpo import VRPO_TARGETS, LoRAMoEPolicy, VRPOTrainer, VRPOTrainingConfig


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


def _expert_policy(seed=0, targets=VRPO_TARGETS):
    cfg = PRESETS["tiny-moe"]
    return LoRAMoEPolicy(build_weights(cfg, random_state_dict(cfg, seed=seed), device="cpu"),
                         LoRAConfig(rank=4, targets=targets))


def test_expert_adapters_default_targets_and_gradients():
    cfg = PRESETS["tiny-moe"]
    pol = LoRAMoEPolicy(build_weights(cfg, random_state_dict(cfg, seed=0), device="cpu"))
    assert pol.lora.targets == VRPO_TARGETS and pol.lora.dropout == 0.05 and pol.lora.rank == 16
    assert {f"gu{e}" for e in range(cfg.num_experts)} <= set(pol.adapters[0])
    pol = _expert_policy()
    from online_speculation_b200.dllm.vrpo import AdapterDisabledReference

    est = estimate_vrpo_preference_loss(pol, AdapterDisabledReference(pol), prompt=(1, 2, 3), chosen=(4, 5, 6, 7),
                                        rejected=(8, 9, 10, 11), mask_token_id=511,
                                        config=VRPOSamplingConfig(timestep_samples=2), beta=0.1)
    assert float(est.loss) == pytest.approx(math.log(2), abs=1e-6)
    est.loss.backward()
    # B starts at zero, so only the B blocks of routed experts receive gradient at initialisation
    got = 0.0
    for layer in pol.adapters:
        for e in range(cfg.num_experts):
            for key in (f"gu{e}", f"down{e}"):
                a = layer[key]
                off = next(o for (ad, name, o, shape) in pol._views if ad is a and name == "B")
                got += float(pol.flat.grad[off:off + a.B.numel()].abs().sum())
    assert got > 0


def test_expert_adapters_fold_into_merged_weights():
    torch.manual_seed(0)
    pol = _expert_policy(seed=2)
    with torch.no_grad():
        pol.flat.add_(torch.randn_like(pol.flat) * 0.05)      # non-zero B everywhere
    pol.eval()
    tokens = torch.randint(0, 500, (2, 12))
    with torch.no_grad():
        got = pol.hidden(tokens).float()
    merged = LoRAMoEPolicy(pol.merged_weights(), LoRAConfig(rank=4, targets=("o_proj",)))
    merged.eval()
    with torch.no_grad(), merged.disable_adapter():
        want = merged.hidden(tokens).float()
    assert float((got - want).norm() / want.norm()) < 5e-2    # bf16 rounding accumulated over the layers


def test_expert_adapters_layer_matches_folded_weights():
    """One MoE layer: adapted experts == the same experts with W + s (B * mask) A folded in."""
    from online_speculation_b200.training.moe_autograd import FrozenExperts, moe_ffn_lora

    torch.manual_seed(1)
    cfg = PRESETS["tiny-moe"]
    pol = _expert_policy(seed=3)
    with torch.no_grad():
        pol.flat.copy_(torch.randn_like(pol.flat) * 0.05)
    pol.eval()
    pol._refresh_views()
    lw, mlw, ad = pol.w.layers[0], pol.merged_weights().layers[0], pol.adapters[0]
    E = cfg.num_experts
    ex = FrozenExperts(lw.router, lw.w_gu, lw.w_down, cfg.num_experts_per_tok, cfg.norm_topk_prob)
    exm = FrozenExperts(mlw.router, mlw.w_gu, mlw.w_down, cfg.num_experts_per_tok, cfg.norm_topk_prob)
    x = torch.randn(16, cfg.hidden_size).bfloat16()
    h = torch.zeros(16, cfg.hidden_size).bfloat16()
    with torch.no_grad():
        a = moe_ffn_lora(x, h, ex, [ad[f"gu{e}"] for e in range(E)], [ad[f"down{e}"] for e in range(E)],
                         pol.lora.scale).float()
        b = moe_ffn_lora(x, h, exm, [None] * E, [None] * E, pol.lora.scale).float()
    assert float((a - b).norm() / b.norm()) < 1.5e-2


def test_expert_gate_only_target_masks_up_rows():
    pol = _expert_policy(targets=("gate_proj",))
    a = pol.adapters[0]["gu0"]
    rows = torch.arange(a.block_mask.shape[0])
    up = (rows % 128) >= 64
    assert float(a.block_mask[up].abs().sum()) == 0 and float(a.block_mask[~up][:, :4].min()) == 1
    assert "down0" not in pol.adapters[0] and "qkv" not in pol.adapters[0]


def test_policy_elbo_with_classifier_free_guidance_matches_full_logits():
    from online_speculation_b200.training.vrpo import _rms

    pol = _policy(seed=4)
    with torch.no_grad():
        pol.flat.add_(torch.randn_like(pol.flat) * 0.05)
    pol.eval()

    class Full:
        """The same policy exposed as full-vocabulary logits (the generic ELBO path)."""

        def parameters(self):
            return iter([pol.flat])

        def __call__(self, t):
            class O:
                pass
            o = O()
            B, L = t.shape
            h = _rms(pol.hidden(t), pol.w.final_norm, pol.cfg.rms_norm_eps)
            o.logits = (h.float() @ pol.w.head.float().t()).view(B, L, -1)
            return o

    plan = sample_vrpo_mask_plan(5, VRPOSamplingConfig(timestep_samples=3), np.random.default_rng(2))
    kw = dict(prompt=(1, 2, 3), answer=(4, 5, 6, 7, 8), mask_token_id=511, plan=plan, cfg_scale=1.5)
    got = estimate_masked_elbo(pol, **kw)
    want = estimate_masked_elbo(Full(), **kw)
    assert float(got) == pytest.approx(float(want), rel=2e-2)
    assert float(got) != pytest.approx(float(estimate_masked_elbo(pol, **dict(kw, cfg_scale=0.0))), rel=1e-4)
    got.backward()
    assert torch.isfinite(pol.flat.grad).all() and pol.flat.grad.abs().sum() > 0
