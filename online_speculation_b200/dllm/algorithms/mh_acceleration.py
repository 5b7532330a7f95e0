"""Exact accelerations of whole-continuation diffusion MH.

Reference behaviour: src/inference_scaling/dllm/algorithms/mh_acceleration.py:56-323.

* Delayed acceptance: a cheap surrogate reward screens proposals (stage one);
  only survivors pay for the exact reward, and stage two accepts with the
  ratio of exp((r - s) / tau) so the chain still targets p exp(r / tau).
* Replay mixture: the independence proposal is the mixture
  (1 - h) q_base + h * empirical(frozen cache); proposal densities use the
  exact trajectory log-probability and the cache's empirical frequency of the
  identical trajectory (same tokens and commit trace).
"""

from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from math import isfinite, log
from typing import Hashable, Sequence

import numpy as np

from ...shared.mh import decide_metropolis_hastings
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import DiffusionMHConfig, DiffusionSamplingConfig
from ..types import DiffusionBackend, DiffusionSample
from .mh import mh_requests, mh_rewards, sample_in_batches


@dataclass(frozen=True, slots=True)
class DelayedDiffusionMHStep:
    update: int
    stage_one_accepted: bool
    exact_reward_evaluated: bool
    accepted: bool
    stage_one_log_acceptance: float
    stage_two_log_acceptance: float | None


@dataclass(frozen=True, slots=True)
class DelayedDiffusionMHResult:
    prompt: TokenSequence
    initial: DiffusionSample
    final: DiffusionSample
    final_reward: float
    final_surrogate_reward: float
    steps: tuple[DelayedDiffusionMHStep, ...]
    exact_reward_evaluations: int
    surrogate_reward_evaluations: int

    @property
    def acceptance_rate(self) -> float:
        return sum(s.accepted for s in self.steps) / len(self.steps) if self.steps else 0.0


def run_diffusion_reward_mh_delayed(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionMHConfig,
                                    sampling: DiffusionSamplingConfig, reward=None, reward_batch=None,
                                    surrogate_reward=None, surrogate_reward_batch=None,
                                    proposal_batch_size: int | None = None, seed: int = 0
                                    ) -> DelayedDiffusionMHResult:
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one exact reward callback")
    if (surrogate_reward is None) == (surrogate_reward_batch is None):
        raise ValueError("provide exactly one surrogate reward callback")
    sampling.validate_generation_length(config.total_length, prefix_length=len(prompt))
    tau = config.reward_temperature
    seeds = SeedStream(seed)
    samples = sample_in_batches(backend, mh_requests(prompt, config, sampling, seeds), proposal_batch_size)
    sur = mh_rewards(prompt, samples, surrogate_reward, surrogate_reward_batch)
    cur, cur_s = samples[0], sur[0]
    cur_r = mh_rewards(prompt, (cur,), reward, reward_batch)[0]
    exact, steps = 1, []
    for u, (prop, ps) in enumerate(zip(samples[1:], sur[1:]), start=1):
        one = decide_metropolis_hastings(current_target_log_density=cur_s / tau, proposed_target_log_density=ps / tau,
                                         uniform=float(seeds.generator("dllm-mh", "delayed", u, "stage-one").random()))
        two_log, accepted, pr = None, False, None
        if one.accepted:
            pr = mh_rewards(prompt, (prop,), reward, reward_batch)[0]
            exact += 1
            two = decide_metropolis_hastings(
                current_target_log_density=(cur_r - cur_s) / tau, proposed_target_log_density=(pr - ps) / tau,
                uniform=float(seeds.generator("dllm-mh", "delayed", u, "stage-two").random()))
            two_log, accepted = two.log_acceptance, two.accepted
        if accepted:
            cur, cur_r, cur_s = prop, pr, ps
        steps.append(DelayedDiffusionMHStep(u, one.accepted, one.accepted, accepted, one.log_acceptance, two_log))
    return DelayedDiffusionMHResult(prompt, samples[0], cur, cur_r, cur_s, tuple(steps), exact, len(samples))


def trajectory_key(sample: DiffusionSample) -> Hashable:
    return sample.token_ids, tuple((s.block_index, s.step_index, s.positions, s.token_ids) for s in sample.trace)


@dataclass(frozen=True, slots=True)
class ReplayMixtureDiffusionMHStep:
    update: int
    proposal_source: str
    accepted: bool
    log_acceptance: float


@dataclass(frozen=True, slots=True)
class ReplayMixtureDiffusionMHResult:
    prompt: TokenSequence
    final: DiffusionSample
    final_reward: float
    steps: tuple[ReplayMixtureDiffusionMHStep, ...]
    base_draws: int
    history_draws: int

    @property
    def acceptance_rate(self) -> float:
        return sum(s.accepted for s in self.steps) / len(self.steps) if self.steps else 0.0


def run_diffusion_replay_mixture_mh(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionMHConfig,
                                    sampling: DiffusionSamplingConfig, history: Sequence[DiffusionSample],
                                    history_probability: float, reward=None, reward_batch=None, seed: int = 0
                                    ) -> ReplayMixtureDiffusionMHResult:
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one reward callback")
    h = float(history_probability)
    if not 0 <= h < 1:
        raise ValueError("history_probability must lie in [0, 1)")
    if h > 0 and not history:
        raise ValueError("positive history probability requires a frozen cache")
    if not sampling.has_exact_trajectory_density:
        raise ValueError("replay-mixture MH requires exact trajectory probabilities")
    for s in history:
        if (s.prefix != prompt or s.trajectory_logprob is None or s.policy_id != sampling.policy_id
                or s.model_id != backend.model_id):
            raise ValueError("cached trajectories must match the prompt and exact policy")
    seeds = SeedStream(seed)
    use_hist = [False] + [bool(v) for v in seeds.generator("dllm-replay-mh", "sources").random(config.updates) < h]
    reqs = mh_requests(prompt, config, sampling, seeds)
    base_idx = [i for i, c in enumerate(use_hist) if not c]
    drawn = dict(zip(base_idx, sample_in_batches(backend, [reqs[i] for i in base_idx], None)))
    for i, c in enumerate(use_hist):
        if c:
            drawn[i] = history[int(seeds.generator("dllm-replay-mh", "history", i).integers(len(history)))]
    samples = [drawn[i] for i in range(config.updates + 1)]
    rewards = mh_rewards(prompt, samples, reward, reward_batch)
    counts = Counter(trajectory_key(s) for s in history)

    def q(s: DiffusionSample) -> float:
        if s.trajectory_logprob is None:
            raise ValueError("an MH proposal omitted its trajectory probability")
        if h == 0:
            return float(s.trajectory_logprob)
        c = counts.get(trajectory_key(s), 0)
        emp = log(c / len(history)) if c else float("-inf")
        return float(np.logaddexp(log(1 - h) + s.trajectory_logprob, log(h) + emp))

    tau = config.reward_temperature
    cur, cur_r = samples[0], rewards[0]
    cur_q = q(cur)
    steps = []
    for u, (prop, pr, c) in enumerate(zip(samples[1:], rewards[1:], use_hist[1:]), start=1):
        pq = q(prop)
        d = decide_metropolis_hastings(current_target_log_density=cur.trajectory_logprob + cur_r / tau,
                                       proposed_target_log_density=prop.trajectory_logprob + pr / tau,
                                       forward_proposal_log_probability=pq, reverse_proposal_log_probability=cur_q,
                                       uniform=float(seeds.generator("dllm-replay-mh", "accept", u).random()))
        if d.accepted:
            cur, cur_r, cur_q = prop, pr, pq
        steps.append(ReplayMixtureDiffusionMHStep(u, "history" if c else "base", d.accepted, d.log_acceptance))
    if not isfinite(cur_r):
        raise ValueError("reward must be finite")
    return ReplayMixtureDiffusionMHResult(prompt, cur, cur_r, tuple(steps), len(base_idx), sum(use_hist))


__all__ = ["DelayedDiffusionMHResult", "DelayedDiffusionMHStep", "ReplayMixtureDiffusionMHResult",
           "ReplayMixtureDiffusionMHStep", "run_diffusion_replay_mixture_mh", "run_diffusion_reward_mh_delayed",
           "trajectory_key"]
