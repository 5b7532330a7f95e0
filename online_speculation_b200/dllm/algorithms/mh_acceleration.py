"""Exact accelerations of whole-continuation diffusion MH.

* Delayed acceptance: a cheap surrogate reward s screens proposals first; only
  proposals that pass pay for the exact reward r, and the second stage accepts with
  exp(((r' - s') - (r - s)) / tau), so the chain still targets p exp(r / tau).
* Replay mixture: the independence proposal is (1 - h) q_base + h * empirical(frozen
  cache); a proposal's density combines its exact trajectory log-probability with the
  cache's frequency of the identical trajectory (tokens and commit trace).

Both precompute every state-independent quantity (draws, surrogate rewards, mixture
densities) as arrays before walking the chain.  Stream names follow
src/inference_scaling/dllm/algorithms/mh_acceleration.py.
"""

from __future__ import annotations

from collections import Counter
from dataclasses import dataclass
from typing import Hashable, Sequence

import numpy as np

from ...shared.mh import mh_accept_batch, mh_log_acceptance_batch
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import DiffusionMHConfig, DiffusionSamplingConfig
from ..types import DiffusionBackend, DiffusionSample
from .mh import mh_requests, mh_rewards, sample_in_batches


def _one_callback(single, batch, what: str) -> None:
    if (single is None) == (batch is None):
        raise ValueError(f"give exactly one {what} callback (single or batched)")


def _uniform(seeds: SeedStream, *name) -> float:
    return float(seeds.generator(*name).random())


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
    _one_callback(reward, reward_batch, "exact reward")
    _one_callback(surrogate_reward, surrogate_reward_batch, "surrogate reward")
    sampling.validate_generation_length(config.total_length, prefix_length=len(prompt))
    tau = config.reward_temperature
    seeds = SeedStream(seed)
    draws = sample_in_batches(backend, mh_requests(prompt, config, sampling, seeds), proposal_batch_size)
    surrogate = np.asarray(mh_rewards(prompt, draws, surrogate_reward, surrogate_reward_batch))

    def exact(i: int) -> float:
        return mh_rewards(prompt, (draws[i],), reward, reward_batch)[0]

    state, state_reward = 0, exact(0)
    evaluations = 1
    steps = []
    for u in range(1, len(draws)):
        first = mh_log_acceptance_batch(surrogate[state] / tau, surrogate[u] / tau)
        passed = bool(mh_accept_batch(first, _uniform(seeds, "dllm-mh", "delayed", u, "stage-one")))
        second, accepted = None, False
        if passed:
            proposed_reward = exact(u)
            evaluations += 1
            second = mh_log_acceptance_batch((state_reward - surrogate[state]) / tau,
                                             (proposed_reward - surrogate[u]) / tau)
            accepted = bool(mh_accept_batch(second, _uniform(seeds, "dllm-mh", "delayed", u, "stage-two")))
            if accepted:
                state, state_reward = u, proposed_reward
        steps.append(DelayedDiffusionMHStep(u, passed, passed, accepted, float(first),
                                            None if second is None else float(second)))
    return DelayedDiffusionMHResult(prompt, draws[0], draws[state], state_reward, float(surrogate[state]),
                                    tuple(steps), evaluations, len(draws))


def trajectory_key(sample: DiffusionSample) -> Hashable:
    """Identity of a trajectory: final tokens and the full commit trace."""
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


def _check_cache(history, prompt, sampling, backend) -> None:
    for s in history:
        if (s.prefix != prompt or s.trajectory_logprob is None or s.policy_id != sampling.policy_id
                or s.model_id != backend.model_id):
            raise ValueError("every cached trajectory must come from this prompt, policy and model, with its density")


def run_diffusion_replay_mixture_mh(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionMHConfig,
                                    sampling: DiffusionSamplingConfig, history: Sequence[DiffusionSample],
                                    history_probability: float, reward=None, reward_batch=None, seed: int = 0
                                    ) -> ReplayMixtureDiffusionMHResult:
    _one_callback(reward, reward_batch, "reward")
    h = float(history_probability)
    if not 0.0 <= h < 1.0:
        raise ValueError("history_probability must lie in [0, 1)")
    if h > 0 and not history:
        raise ValueError("a positive history probability needs a frozen cache")
    if not sampling.has_exact_trajectory_density:
        raise ValueError("the mixture density needs exact trajectory probabilities")
    _check_cache(history, prompt, sampling, backend)
    seeds = SeedStream(seed)
    from_cache = np.concatenate(([False], seeds.generator("dllm-replay-mh", "sources").random(config.updates) < h))
    requests = mh_requests(prompt, config, sampling, seeds)
    fresh = np.flatnonzero(~from_cache)
    draws: list = [None] * len(requests)
    for i, s in zip(fresh, sample_in_batches(backend, [requests[i] for i in fresh], None)):
        draws[i] = s
    for i in np.flatnonzero(from_cache):
        pick = int(seeds.generator("dllm-replay-mh", "history", int(i)).integers(len(history)))
        draws[i] = history[pick]
    rewards = np.asarray(mh_rewards(prompt, draws, reward, reward_batch))
    if any(s.trajectory_logprob is None for s in draws):
        raise ValueError("an MH proposal came without its trajectory probability")
    base = np.asarray([s.trajectory_logprob for s in draws], dtype=np.float64)
    if h == 0:
        proposal = base
    else:
        frequency = Counter(trajectory_key(s) for s in history)
        with np.errstate(divide="ignore"):
            empirical = np.log(np.asarray([frequency.get(trajectory_key(s), 0) for s in draws]) / len(history))
        proposal = np.logaddexp(np.log1p(-h) + base, np.log(h) + empirical)
    target = base + rewards / config.reward_temperature
    state = 0
    steps = []
    for u in range(1, len(draws)):
        log_a = mh_log_acceptance_batch(target[state], target[u], proposal[u], proposal[state])
        accepted = bool(mh_accept_batch(log_a, _uniform(seeds, "dllm-replay-mh", "accept", u)))
        if accepted:
            state = u
        steps.append(ReplayMixtureDiffusionMHStep(u, "history" if from_cache[u] else "base", accepted, float(log_a)))
    if not np.isfinite(rewards[state]):
        raise ValueError("rewards have to be finite")
    return ReplayMixtureDiffusionMHResult(prompt, draws[state], float(rewards[state]), tuple(steps), int(fresh.size),
                                          int(from_cache.sum()))


__all__ = ["DelayedDiffusionMHResult", "DelayedDiffusionMHStep", "ReplayMixtureDiffusionMHResult",
           "ReplayMixtureDiffusionMHStep", "run_diffusion_replay_mixture_mh", "run_diffusion_reward_mh_delayed",
           "trajectory_key"]
