"""Cold-start service: budget admission, learning, paired publication trials and resume (CPU)."""

import pytest
import torch

from online_speculation_b200.blockspec.cold_start import (CleanReplay, ColdStartService, ServiceConfig,
                                                          TimeBudget)
from online_speculation_b200.blockspec.fitting import FitConfig
from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder

CFG = DualViewConfig(vocab_size=17, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=4, block_size=4, mask_token_id=1)


def _model():
    torch.manual_seed(0)
    return DualViewDecoder(CFG).eval().requires_grad_(False)


def test_time_budget_admission_and_debt():
    b = TimeBudget(0.1)
    assert not b.admits(0.5)
    b.delivered(10.0)
    assert b.admits(0.5) and b.credit == pytest.approx(1.0)
    b.charge("training", 1.5)
    assert not b.admits(0.1) and b.summary()["debt_seconds"] == pytest.approx(0.5)
    with pytest.raises(ValueError):
        TimeBudget(0.5)


def test_clean_replay_batches_are_deterministic():
    r1, r2 = CleanReplay(4, 8, 4, seed=3), CleanReplay(4, 8, 4, seed=3)
    for r in (r1, r2):
        r.append(torch.arange(12)[None])
        r.append(torch.arange(3)[None])       # shorter than a block: dropped
    assert len(r1.records) == 1
    a, b = r1.batch(2, 2), r2.batch(2, 2)
    assert all(torch.equal(x[0], y[0]) and torch.equal(x[1], y[1]) for x, y in zip(a, b))
    assert a[0][0].shape == (1, 8)


def test_service_learns_probes_and_resumes():
    fit = FitConfig(steps=50, sequence_length=16, anchors_per_sequence=2, warmup_steps=1, learning_rate=1e-2)
    cfg = ServiceConfig(fraction=0.1, replay_records=8, probe_every=2, probe_tokens=6, publish_margin=1.01,
                        initial_step_estimate=1e-4, initial_probe_factor=1.0)
    gate = [torch.tensor([[3, 4, 5, 6]])]
    svc = ColdStartService(_model(), fit, cfg, gate_prompts=gate)
    draft0 = {n: p.clone() for n, p in svc.learner.execution.items()}
    # pre-earned credit (as if 100 s and 100k tokens had been served) so that training and probes are admitted
    svc.budget.delivered(100.0)
    svc.tokens = 100_000
    probes = []
    for i in range(6):
        out, info = svc.serve(torch.tensor([[2 + i, 3, 4]]), 12, seed=i)
        assert len(out.tokens) == 12 and info["request"] == i + 1 and info["mode"] in ("ar", "speculative")
        if info["probe"] is not None:
            probes.append(info["probe"])
    assert svc.learner.steps >= 2 and probes and all("paired_ratios" in p for p in probes)
    # serving weights only change on publication
    if svc.learner.serving_step == 0:
        assert all(torch.equal(p, draft0[n]) for n, p in svc.learner.execution.items())
    state = svc.state_dict()
    fresh = ColdStartService(_model(), fit, cfg, gate_prompts=gate)
    fresh.load_state_dict(state)
    assert fresh.learner.steps == svc.learner.steps and len(fresh.replay.records) == len(svc.replay.records)
    assert all(torch.equal(fresh.learner.master[n], svc.learner.master[n]) for n in svc.learner.master)
    assert fresh.budget.costs.get("resume", 0) >= 0
    with pytest.raises(ValueError):
        ColdStartService(_model(), fit, cfg, gate_prompts=[torch.tensor([[9, 9, 9, 9]])]).load_state_dict(state)


def _run_live(cfg, requests=8, max_new=12):
    fit = FitConfig(steps=50, sequence_length=16, anchors_per_sequence=2, warmup_steps=1, learning_rate=1e-2)
    gate = [torch.tensor([[3, 4, 5, 6]])]
    svc = ColdStartService(_model(), fit, cfg, gate_prompts=gate)
    svc.budget.delivered(100.0)
    svc.tokens = 100_000
    probes = []
    for i in range(requests):
        out, info = svc.serve(torch.tensor([[2 + i, 3, 4]]), max_new, seed=i)
        assert len(out.tokens) == max_new
        if info["probe"] is not None:
            probes.append(info["probe"])
    return svc, fit, gate, probes


def test_live_ar_prefix_trials_pool_and_resume():
    cfg = ServiceConfig(fraction=0.1, replay_records=8, probe_every=2, probe_tokens=6, publish_margin=1.01,
                        initial_step_estimate=1e-4, initial_probe_factor=1.0, reuse_ar_prefix=True,
                        live_probe_requests=2)
    svc, fit, gate, probes = _run_live(cfg)
    live = [p for p in probes if p.get("reference_kind") == "delivered_ar_prefix"]
    # records carry the pooled totals of the trials so far
    assert live and all(p["reference_tokens"] == 6 * p["probe_requests"] and p["reference_seconds"] > 0
                        for p in live)
    assert any(p["probe_requests"] == 2 and p["complete"] for p in live)
    assert all(not p["passed"] for p in live if not p["complete"])
    fresh = ColdStartService(_model(), fit, cfg, gate_prompts=gate)
    fresh.load_state_dict(svc.state_dict())
    assert fresh.pending_live == svc.pending_live
    with pytest.raises(ValueError):
        ServiceConfig(reuse_ar_prefix=True, full_answer_screen=True)
    with pytest.raises(ValueError):
        ServiceConfig(live_probe_requests=2)
    with pytest.raises(ValueError):
        ColdStartService(_model(), fit, cfg)            # trials after publication need gate prompts


def test_full_answer_screen_then_confirmation_and_resume():
    cfg = ServiceConfig(fraction=0.1, replay_records=8, probe_every=2, probe_tokens=6, publish_margin=1.01,
                        initial_step_estimate=1e-4, initial_probe_factor=1.0, full_answer_screen=True,
                        screen_requests=1, screen_margin=1.0, initial_screen_estimate=1e-3)
    svc, fit, gate, probes = _run_live(cfg, requests=10)
    screens = [p for p in probes if p.get("stage") == "screen"]
    assert screens and all(p["predicted_seconds"] > 0 and p["virtual_forwards"] > 0 for p in screens)
    assert all(p["reference_kind"] in ("delivered_ar_full", "delivered_speculative_full") for p in screens)
    # a screen either awaits its confirmation or was discarded; confirmations decide publication
    for p in screens:
        assert p["awaiting_confirmation"] or p["complete"]
    confirmations = [p for p in probes if p.get("stage") == "confirmation"]
    assert all(p["complete"] and "candidate_over_ar" in p for p in confirmations)
    if any(p["passed"] for p in confirmations):
        assert svc.learner.serving_step > 0
    state = svc.state_dict()
    fresh = ColdStartService(_model(), fit, cfg, gate_prompts=gate)
    fresh.load_state_dict(state)
    assert fresh.full_gate.state_dict() == svc.full_gate.state_dict()
    other = ServiceConfig(fraction=0.1, replay_records=8, probe_every=2, probe_tokens=6, publish_margin=1.01,
                          initial_step_estimate=1e-4, initial_probe_factor=1.0)
    with pytest.raises(ValueError):
        ColdStartService(_model(), fit, other, gate_prompts=gate).load_state_dict(state)
