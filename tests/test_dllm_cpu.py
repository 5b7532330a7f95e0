"""dLLM layer on CPU: configs, the block-diffusion backend on a tiny module, and every algorithm
on a fake Bernoulli-token diffusion backend with exact trajectory densities."""

import itertools
import math

import numpy as np
import pytest
import torch

from online_speculation_b200.dllm import (DiffusionEngineBackend, DiffusionGenerationRequest, DiffusionISConfig,
                                          DiffusionMHConfig, DiffusionSample, DiffusionSamplingConfig,
                                          DiffusionTraceStep, DiffusionTrajectoryScoreRequest, ModuleLogits,
                                          diffusion_decision_stage_lengths)
from online_speculation_b200.dllm.algorithms import (resample_diffusion_candidates, run_conditional_diffusion_is,
                                                     run_diffusion_block_beam, run_diffusion_replay_mixture_mh,
                                                     run_diffusion_reward_mh, run_diffusion_reward_mh_delayed,
                                                     run_diffusion_smc_rollout_forest,
                                                     run_diffusion_trajectory_power_mh,
                                                     run_progressive_diffusion_is)
from online_speculation_b200.dllm.config import DiffusionBlockBeamConfig, DiffusionPowerMHConfig
from online_speculation_b200.dllm.dynamic_is import run_dynamic_diffusion_is
from online_speculation_b200.shared.config import SMCForestConfig


# ------------------------------------------------------------------ configs --
def test_decision_stages_keep_whole_blocks():
    sp = DiffusionSamplingConfig(block_length=8, steps_per_block=4)
    assert diffusion_decision_stage_lengths(prompt_length=3, total_length=32, decision_block_size=16,
                                            sampling=sp) == (16, 16)
    with pytest.raises(ValueError):
        diffusion_decision_stage_lengths(prompt_length=0, total_length=32, decision_block_size=12, sampling=sp)
    with pytest.raises(ValueError):
        DiffusionGenerationRequest((1,), 12, sp, 0, "x")


def test_policy_id_and_exactness():
    sp = DiffusionSamplingConfig(temperature=0.5, remasking="random", mask_token_id=7)
    assert sp.policy_id == ("block=32;steps=32;temperature=0.5;top_k=0;top_p=1.0;cfg=0.0;remasking=random;"
                            "threshold=0.85;mask=7")
    assert DiffusionSamplingConfig(temperature=1.0000001).policy_id != \
        DiffusionSamplingConfig(temperature=1.0000002).policy_id
    for bad in ({"temperature": float("nan")}, {"top_p": float("inf")}, {"cfg_scale": float("nan")}):
        with pytest.raises(ValueError):
            DiffusionSamplingConfig(**bad)
    assert sp.has_exact_trajectory_density
    assert not DiffusionSamplingConfig(temperature=0.5).has_exact_trajectory_density
    assert DiffusionSamplingConfig(block_length=5, steps_per_block=2).transfer_schedule() == (3, 2)
    with pytest.raises(ValueError):
        DiffusionSamplingConfig(block_length=4, steps_per_block=5)


def test_exact_trace_must_be_complete_and_consistent():
    step = DiffusionTraceStep(0, 0, (0, 1), (3, 4), -1.0)
    DiffusionSample((), (3, 4), (step,), -1.0, "p", "m", "r")
    with pytest.raises(ValueError):
        DiffusionSample((), (3, 5), (step,), -1.0, "p", "m", "r")
    with pytest.raises(ValueError):
        DiffusionSample((), (3, 4), (step,), -2.0, "p", "m", "r")


# ------------------------------------------------------------------ backend --
class TinyBidirectional(torch.nn.Module):
    def __init__(self, V=13, H=16, layers=2):
        super().__init__()
        self.emb = torch.nn.Embedding(V, H)
        self.mix = torch.nn.ModuleList(torch.nn.Linear(H, H) for _ in range(layers))
        self.out = torch.nn.Linear(H, V)

    def forward(self, t):
        x = self.emb(t)
        for m in self.mix:
            x = x + torch.tanh(m(x.mean(1, keepdim=True)))
        return self.out(x)


def _backend(**kw):
    torch.manual_seed(0)
    return DiffusionEngineBackend(ModuleLogits(TinyBidirectional(), mask_token_id=12), model_id="tiny", **kw)


def test_random_remasking_trace_rescores_to_its_probability():
    be = _backend()
    sp = DiffusionSamplingConfig(block_length=4, steps_per_block=2, temperature=0.8, remasking="random")
    reqs = [DiffusionGenerationRequest((1, 2, 3), 8, sp, seed=s, request_id=str(s)) for s in range(3)]
    out = be.sample_batch(reqs)
    scores = be.score_trajectories([DiffusionTrajectoryScoreRequest(s, sp) for s in out])
    for s, v in zip(out, scores):
        assert s.trajectory_logprob == pytest.approx(v, abs=1e-9)
        assert all(t != 12 for t in s.token_ids)          # the mask token is never committed
    hot = DiffusionSamplingConfig(block_length=4, steps_per_block=2, temperature=2.0, remasking="random")
    other = be.score_trajectories([DiffusionTrajectoryScoreRequest(out[0], hot)])[0]
    assert other != pytest.approx(scores[0])


def test_low_confidence_is_not_labelled_exact_and_greedy_is_deterministic():
    be = _backend()
    sp = DiffusionSamplingConfig(block_length=4, steps_per_block=4, temperature=0.0)
    a = be.sample_batch([DiffusionGenerationRequest((1,), 8, sp, 0, "a")])[0]
    b = be.sample_batch([DiffusionGenerationRequest((1,), 8, sp, 5, "b")])[0]
    assert a.trajectory_logprob is None and a.token_ids == b.token_ids
    with pytest.raises(ValueError):
        be.score_trajectories([DiffusionTrajectoryScoreRequest(a, sp)])


def test_batch_limit_does_not_change_samples():
    sp = DiffusionSamplingConfig(block_length=4, steps_per_block=2, temperature=1.0, remasking="sequential")
    reqs = [DiffusionGenerationRequest((2, 3), 8, sp, seed=s, request_id=str(s)) for s in range(4)]
    full = _backend().sample_batch(reqs)
    chunked = _backend(max_batch_size=1).sample_batch(reqs)
    assert [s.token_ids for s in full] == [s.token_ids for s in chunked]
    assert [s.trajectory_logprob for s in full] == pytest.approx([s.trajectory_logprob for s in chunked])


def test_cfg_and_snapshot():
    be = _backend()
    sp = DiffusionSamplingConfig(block_length=4, steps_per_block=4, temperature=0.0, cfg_scale=1.5)
    be.sample_batch([DiffusionGenerationRequest((4, 5), 4, sp, 0, "x")])
    snap = be.snapshot()
    assert snap.forward_calls == 4 and snap.model_sequences == 8 and snap.generated_tokens == 4
    assert be.with_prefix_layers(1).model_id == "tiny#prefix-layers=1"


# ------------------------------------------------------- fake coin backend --
class CoinBackend:
    """Tokens are iid Bernoulli(theta) per position; the trace commits one position per step in order."""

    def __init__(self, theta=0.3, model_id="coin"):
        self.theta, self._id = theta, model_id
        self.sample_calls = 0

    @property
    def model_id(self):
        return self._id

    def _trace(self, toks, sp, theta):
        steps, bl = [], sp.block_length
        sched = sp.transfer_schedule()
        pos = 0
        for b in range(len(toks) // bl):
            for k, n in enumerate(sched):
                ps = tuple(range(pos, pos + n))
                lp = sum(math.log(theta if toks[p] else 1 - theta) for p in ps)
                steps.append(DiffusionTraceStep(b, k, ps, tuple(toks[p] for p in ps), lp))
                pos += n
        return tuple(steps)

    def sample_batch(self, reqs):
        self.sample_calls += 1
        out = []
        for r in reqs:
            rng = np.random.default_rng(r.seed)
            toks = tuple(int(v) for v in rng.random(r.generation_length) < self.theta)
            tr = self._trace(toks, r.sampling, self.theta)
            out.append(DiffusionSample(r.prefix, toks, tr, sum(s.logprob for s in tr), r.sampling.policy_id,
                                       self._id, r.request_id))
        return out

    def score_trajectories(self, reqs):
        return [sum(math.log(self.theta if t else 1 - self.theta) for t in r.sample.token_ids) for r in reqs]


EXACT = DiffusionSamplingConfig(block_length=2, steps_per_block=2, temperature=1.0, remasking="sequential")


def reward_ones(prompt, cont):
    return float(sum(cont))


def reward_batch(prompt, conts):
    return [float(sum(c)) for c in conts]


def test_independence_mh_targets_base_times_exp_reward():
    be = CoinBackend(0.3)
    res = run_diffusion_reward_mh(backend=be, prompt=(9,), config=DiffusionMHConfig(total_length=2, updates=4000,
                                                                                    reward_temperature=1.0),
                                  sampling=EXACT, reward=reward_ones, seed=1, proposal_batch_size=500)
    states = [res.initial.token_ids] + [None] * 0
    cur = res.initial.token_ids
    counts = {}
    for st in res.steps:
        if st.accepted:
            cur = st.proposal.token_ids
        counts[cur] = counts.get(cur, 0) + 1
    exact = {}
    for x in itertools.product((0, 1), repeat=2):
        exact[x] = math.prod(0.3 if v else 0.7 for v in x) * math.exp(sum(x))
    z = sum(exact.values())
    n = sum(counts.values())
    for x, p in exact.items():
        assert abs(counts.get(x, 0) / n - p / z) < 0.04, (x, counts.get(x, 0) / n, p / z)
    assert be.sample_calls == 9   # 4001 draws in batches of 500


def test_delayed_and_replay_mixture_mh_run():
    be = CoinBackend(0.4)
    cfg = DiffusionMHConfig(total_length=4, updates=30)
    d = run_diffusion_reward_mh_delayed(backend=be, prompt=(), config=cfg, sampling=EXACT, reward=reward_ones,
                                        surrogate_reward=lambda p, c: 0.5 * sum(c), seed=0)
    assert d.exact_reward_evaluations <= 31 and d.surrogate_reward_evaluations == 31
    hist = be.sample_batch([DiffusionGenerationRequest((), 4, EXACT, s, f"h{s}") for s in range(5)])
    base = run_diffusion_replay_mixture_mh(backend=be, prompt=(), config=cfg, sampling=EXACT, history=hist,
                                           history_probability=0.0, reward=reward_ones, seed=2)
    mix = run_diffusion_replay_mixture_mh(backend=be, prompt=(), config=cfg, sampling=EXACT, history=hist,
                                          history_probability=0.5, reward=reward_ones, seed=2)
    assert base.history_draws == 0 and mix.history_draws > 0
    other = CoinBackend(0.4, model_id="other")
    with pytest.raises(ValueError):
        run_diffusion_replay_mixture_mh(backend=other, prompt=(), config=cfg, sampling=EXACT, history=hist,
                                        history_probability=0.5, reward=reward_ones)


def test_conditional_is_off_policy_ratio_uses_the_same_trajectory():
    base, prop = CoinBackend(0.3, "p"), CoinBackend(0.6, "q")
    cfg = DiffusionISConfig(candidate_count=3, rollout_count=2, block_size=2, total_length=4)
    res = run_conditional_diffusion_is(base_backend=base, prompt=(1,), config=cfg, base_sampling=EXACT,
                                       reward=reward_ones, rollout_backend=prop, seed=3)
    assert len(res.token_ids) == 4 and len(res.steps) == 2
    r = res.steps[0].candidates[0].rollouts[0]
    assert r.raw_log_importance_ratio == pytest.approx(r.target_trajectory_logprob - r.proposal_trajectory_logprob)
    assert abs(sum(res.steps[0].probabilities) - 1) < 1e-9
    sir = resample_diffusion_candidates(samples=prop.sample_batch(
        [DiffusionGenerationRequest((), 2, EXACT, s, str(s)) for s in range(4)]), rewards=[0, 1, 2, 1],
        reward_temperature=1.0, rng=np.random.default_rng(0))
    assert 0 <= sir.selected_index < 4 and sir.effective_sample_size > 1


def test_power_mh_beam_smc_progressive_dynamic_run():
    be = CoinBackend(0.5)
    pm = run_diffusion_trajectory_power_mh(backend=be, prompt=(), config=DiffusionPowerMHConfig(
        total_length=4, decision_block_size=2, updates_per_stage=3, alpha=2.0), sampling=EXACT,
        proposal_sampling=EXACT, seed=0)
    assert len(pm.final.token_ids) == 4 and len(pm.steps) == 6
    beam = run_diffusion_block_beam(backend=CoinBackend(0.2), prompt=(), config=DiffusionBlockBeamConfig(
        total_length=4, decision_block_size=2, width=3, branching_factor=2), sampling=EXACT)
    lps = [b.trajectory_logprob for b in beam.beams]
    assert lps == sorted(lps, reverse=True) and len(beam.beams) == 3
    smc = run_diffusion_smc_rollout_forest(backend=be, prompt=(), config=SMCForestConfig(
        particle_count=4, branch_factor=2, rollout_count=2, block_size=2, total_length=6), sampling=EXACT,
        reward_batch=reward_batch, seed=1)
    assert len(smc.token_ids) == 6 and smc.reused_rollouts > 0
    cfg = DiffusionISConfig(candidate_count=3, rollout_count=2, block_size=2, total_length=4)
    prog = run_progressive_diffusion_is(backend=be, prompt=(), config=cfg, sampling=EXACT, reward_batch=reward_batch,
                                        pilot_rollouts_per_candidate=2, evaluation_rollout_budget=6)
    assert len(prog.token_ids) == 4 and prog.steps[0].pilot_rollouts == 6
    for arm in ("base_candidate_fixed", "trajectory_replay_aware_fixed", "trajectory_replay_aware_optimal"):
        dyn = run_dynamic_diffusion_is(arm=arm, target_backend=CoinBackend(0.4, "t"),
                                       auxiliary_backend=CoinBackend(0.6, "a"), prompt=(), config=cfg,
                                       sampling=EXACT, reward_batch=reward_batch, history_rollouts=2,
                                       fresh_rollouts=1, truncation=1.0, seed=4)
        assert len(dyn.token_ids) == 4
        if arm != "base_candidate_fixed":
            assert dyn.rollout_reuse_rate > 0


def test_conditional_diffusion_is_matches_its_exact_finite_candidate_law():
    """Two decision blocks of 2 coin tokens, 2 candidates, 1 rollout: the sampler's own law, enumerated."""
    from online_speculation_b200.shared.metrics import empirical_distribution, total_variation

    theta, tau = 0.35, 0.5
    be = CoinBackend(theta)

    def reward(_p, y):
        return float(y[0]) + 0.5 * float(len(y) > 2 and y[2] == y[0])

    def p_block(b):
        return math.prod(theta if t else 1 - theta for t in b)

    blocks = list(itertools.product((0, 1), repeat=2))
    first = {}
    for c1, c2, y1, y2 in itertools.product(blocks, repeat=4):
        w1, w2 = math.exp(reward((), c1 + y1) / tau), math.exp(reward((), c2 + y2) / tau)
        pr = p_block(c1) * p_block(c2) * p_block(y1) * p_block(y2)
        first[c1] = first.get(c1, 0.0) + pr * w1 / (w1 + w2)
        first[c2] = first.get(c2, 0.0) + pr * w2 / (w1 + w2)
    law = {}
    for a in blocks:
        second = {}
        for d1, d2 in itertools.product(blocks, repeat=2):
            w1, w2 = math.exp(reward((), a + d1) / tau), math.exp(reward((), a + d2) / tau)
            pr = p_block(d1) * p_block(d2)
            second[d1] = second.get(d1, 0.0) + pr * w1 / (w1 + w2)
            second[d2] = second.get(d2, 0.0) + pr * w2 / (w1 + w2)
        for b, q in second.items():
            law[a + b] = first[a] * q
    assert abs(sum(law.values()) - 1) < 1e-12
    cfg = DiffusionISConfig(candidate_count=2, rollout_count=1, block_size=2, total_length=4, reward_temperature=tau)
    runs = [run_conditional_diffusion_is(base_backend=be, prompt=(), config=cfg, base_sampling=EXACT, reward=reward,
                                         seed=s) for s in range(4000)]
    emp = empirical_distribution(tuple(r.token_ids) for r in runs)
    # 16 outcomes, 4000 runs: sampling noise alone gives a TV of about 0.025
    assert total_variation(emp, law) < 0.05
