"""Whole-continuation independence MH for dLLM reward targets p(trace) exp(r / tau).

Reference behaviour: src/inference_scaling/dllm/algorithms/mh.py:99-168.  With
proposals drawn from the base sampler the base trajectory density cancels, so
the acceptance min(1, exp((r' - r) / tau)) needs rewards only.  All
``updates + 1`` draws are independent of the chain state and are sampled in
batches (``proposal_batch_size``) before the sequential accept / reject pass.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from math import isfinite

from ...shared.mh import decide_metropolis_hastings
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import DiffusionMHConfig, DiffusionSamplingConfig
from ..types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample


def mh_requests(prompt: TokenSequence, config: DiffusionMHConfig, sampling: DiffusionSamplingConfig,
                seeds: SeedStream) -> list[DiffusionGenerationRequest]:
    return [DiffusionGenerationRequest(prompt, config.total_length, sampling, seeds.derive("dllm-mh", d),
                                       f"dllm-mh:draw:{d}") for d in range(config.updates + 1)]


def sample_in_batches(backend: DiffusionBackend, requests: Sequence[DiffusionGenerationRequest],
                      batch_size: int | None) -> list[DiffusionSample]:
    if batch_size is not None and batch_size <= 0:
        raise ValueError("proposal_batch_size must be positive when provided")
    n = batch_size or len(requests)
    out: list[DiffusionSample] = []
    for i in range(0, len(requests), n):
        out.extend(backend.sample_batch(requests[i:i + n]))
    if len(out) != len(requests):
        raise RuntimeError("backend returned an invalid number of MH proposals")
    return out


def mh_rewards(prompt, samples, reward, reward_batch) -> list[float]:
    conts = [s.token_ids for s in samples]
    vals = ([float(v) for v in reward_batch(prompt, conts)] if reward_batch is not None
            else [float(reward(prompt, c)) for c in conts])
    if len(vals) != len(samples):
        raise RuntimeError("reward evaluator returned an invalid number of values")
    if not all(isfinite(v) for v in vals):
        raise ValueError("reward values must be finite")
    return vals


@dataclass(frozen=True, slots=True)
class DiffusionMHStep:
    update: int
    proposal: DiffusionSample
    proposal_reward: float
    previous_reward: float
    acceptance_probability: float
    accepted: bool


@dataclass(frozen=True, slots=True)
class DiffusionMHResult:
    prompt: TokenSequence
    initial: DiffusionSample
    initial_reward: float
    steps: tuple[DiffusionMHStep, ...]
    final: DiffusionSample
    final_reward: float

    @property
    def acceptance_rate(self) -> float:
        return sum(s.accepted for s in self.steps) / len(self.steps) if self.steps else 0.0


def run_diffusion_reward_mh(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionMHConfig,
                            sampling: DiffusionSamplingConfig, reward=None, seed: int = 0, reward_batch=None,
                            proposal_batch_size: int | None = None) -> DiffusionMHResult:
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one of reward or reward_batch")
    sampling.validate_generation_length(config.total_length, prefix_length=len(prompt))
    seeds = SeedStream(seed)
    samples = sample_in_batches(backend, mh_requests(prompt, config, sampling, seeds), proposal_batch_size)
    rewards = mh_rewards(prompt, samples, reward, reward_batch)
    cur, cur_r = samples[0], rewards[0]
    steps = []
    for u, (prop, pr) in enumerate(zip(samples[1:], rewards[1:]), start=1):
        d = decide_metropolis_hastings(current_target_log_density=cur_r / config.reward_temperature,
                                       proposed_target_log_density=pr / config.reward_temperature,
                                       uniform=float(seeds.generator("dllm-mh", "accept", u).random()))
        prev = cur_r
        if d.accepted:
            cur, cur_r = prop, pr
        steps.append(DiffusionMHStep(u, prop, pr, prev, d.acceptance_probability, d.accepted))
    return DiffusionMHResult(prompt, samples[0], rewards[0], tuple(steps), cur, cur_r)


__all__ = ["DiffusionMHResult", "DiffusionMHStep", "mh_requests", "mh_rewards", "run_diffusion_reward_mh",
           "sample_in_batches"]
