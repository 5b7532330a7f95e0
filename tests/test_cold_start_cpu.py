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
