"""Independence MH over whole dLLM continuations for reward targets p(trace) exp(r / tau).

Proposals come from the base sampler, so the base trajectory density cancels and
the acceptance min(1, exp((r' - r) / tau)) needs rewards only.  Every one of the
``updates + 1`` draws is independent of the chain, so all of them are generated
first (in batches of ``proposal_batch_size``) and scored in one pass; the chain
then only walks the precomputed rewards with precomputed uniforms.  Stream names
(``("dllm-mh", d)`` draws, ``("dllm-mh", "accept", u)`` uniforms) and request ids
follow src/inference_scaling/dllm/algorithms/mh.py.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np

from ...shared.mh import mh_accept_batch, mh_log_acceptance_batch
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import DiffusionMHConfig, DiffusionSamplingConfig
from ..types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample


def mh_requests(prompt: TokenSequence, config: DiffusionMHConfig, sampling: DiffusionSamplingConfig,
                seeds: SeedStream) -> list[DiffusionGenerationRequest]:
    return [DiffusionGenerationRequest(prompt, config.total_length, sampling, seeds.derive("dllm-mh", draw),
                                       f"dllm-mh:draw:{draw}") for draw in range(config.updates + 1)]


def sample_in_batches(backend: DiffusionBackend, requests: Sequence[DiffusionGenerationRequest],
                      batch_size: int | None) -> list[DiffusionSample]:
    if batch_size is not None and batch_size < 1:
        raise ValueError("proposal_batch_size has to be positive")
    width = batch_size or max(1, len(requests))
    samples: list[DiffusionSample] = []
    for start in range(0, len(requests), width):
        samples.extend(backend.sample_batch(list(requests[start:start + width])))
    if len(samples) != len(requests):
        raise RuntimeError(f"{len(samples)} proposals came back for {len(requests)} requests")
    return samples


def mh_rewards(prompt, samples, reward, reward_batch) -> list[float]:
    continuations = [s.token_ids for s in samples]
    if reward_batch is not None:
        values = np.asarray(list(reward_batch(prompt, continuations)), dtype=np.float64)
    else:
        values = np.asarray([reward(prompt, c) for c in continuations], dtype=np.float64)
    if values.shape != (len(samples),):
        raise RuntimeError(f"{values.size} rewards for {len(samples)} proposals")
    if not np.isfinite(values).all():
        raise ValueError("rewards have to be finite")
    return values.tolist()


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
        raise ValueError("give either reward or reward_batch")
    sampling.validate_generation_length(config.total_length, prefix_length=len(prompt))
    seeds = SeedStream(seed)
    draws = sample_in_batches(backend, mh_requests(prompt, config, sampling, seeds), proposal_batch_size)
    rewards = np.asarray(mh_rewards(prompt, draws, reward, reward_batch))
    uniforms = np.asarray([seeds.generator("dllm-mh", "accept", u).random() for u in range(1, len(draws))])
    tau = config.reward_temperature
    state = 0
    steps = []
    for u in range(1, len(draws)):
        log_a = mh_log_acceptance_batch(rewards[state] / tau, rewards[u] / tau)
        accepted = bool(mh_accept_batch(log_a, uniforms[u - 1]))
        steps.append(DiffusionMHStep(u, draws[u], float(rewards[u]), float(rewards[state]), float(np.exp(log_a)),
                                     accepted))
        if accepted:
            state = u
    return DiffusionMHResult(prompt, draws[0], float(rewards[0]), tuple(steps), draws[state], float(rewards[state]))


__all__ = ["DiffusionMHResult", "DiffusionMHStep", "mh_requests", "mh_rewards", "run_diffusion_reward_mh",
           "sample_in_batches"]
