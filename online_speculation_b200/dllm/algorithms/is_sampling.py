"""Reward reweighting (SIR) and blockwise conditional importance sampling for masked dLLMs.

Reference behaviour: src/inference_scaling/dllm/algorithms/is_sampling.py:60-533.
Conditional IS commits one decision block at a time: ``candidate_count`` base
candidates are drawn for the block, each is completed by ``rollout_count``
full rollouts, a candidate's log-weight is logmeanexp over its rollouts of
r / tau (+ the trajectory log-ratio log p_target(trace) - log q(trace) when the
rollouts come from another model or transition policy), and one candidate is
drawn from the normalised weights.  Decision blocks never split a native
diffusion block.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import Callable

import numpy as np

from ...shared.importance import MonteCarloRolloutWeightProvider, RolloutObservation
from ...shared.metrics import importance_effective_sample_size
from ...shared.rng import SeedStream
from ...shared.stepwise import StepwiseCandidate, normalize_log_weights, run_stepwise_generation
from ...shared.types import TokenSequence
from ..config import DiffusionISConfig, DiffusionSamplingConfig, diffusion_decision_stage_lengths
from ..types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample, DiffusionTrajectoryScoreRequest

DiffusionRewardFunction = Callable[[TokenSequence, TokenSequence], float]
DiffusionRewardBatchFunction = Callable[[TokenSequence, Sequence[TokenSequence]], Sequence[float]]


@dataclass(frozen=True, slots=True)
class DiffusionSIRItem:
    sample: DiffusionSample
    reward: float
    target_trajectory_logprob: float | None
    raw_log_importance_ratio: float | None
    applied_log_importance_ratio: float | None
    log_weight: float


@dataclass(frozen=True, slots=True)
class DiffusionSIRResult:
    items: tuple[DiffusionSIRItem, ...]
    probabilities: tuple[float, ...]
    selected_index: int
    effective_sample_size: float

    @property
    def selected(self) -> DiffusionSIRItem:
        return self.items[self.selected_index]


def resample_diffusion_candidates(*, samples: Sequence[DiffusionSample], rewards: Sequence[float],
                                  reward_temperature: float, rng: np.random.Generator,
                                  target_trajectory_logprobs: Sequence[float] | None = None,
                                  importance_log_ratio_clip: float | None = None) -> DiffusionSIRResult:
    """Draw one sample from reward-tilted weights (on-policy, or with trajectory IS ratios)."""
    if not samples or len(samples) != len(rewards):
        raise ValueError("samples and rewards must have the same positive length")
    if reward_temperature <= 0:
        raise ValueError("reward_temperature must be positive")
    off = target_trajectory_logprobs is not None
    if off and len(target_trajectory_logprobs) != len(samples):
        raise ValueError("one target trajectory score is required per sample")
    provider = MonteCarloRolloutWeightProvider(reward_temperature=reward_temperature,
                                               correction="importance" if off else "none",
                                               log_ratio_clip=importance_log_ratio_clip if off else None)
    items = []
    for i, (s, r) in enumerate(zip(samples, rewards)):
        tgt = None
        if off:
            if s.trajectory_logprob is None:
                raise ValueError("off-policy IS requires an exact proposal trajectory density")
            tgt = float(target_trajectory_logprobs[i])
        w = provider.weight(RolloutObservation(float(r), tgt, s.trajectory_logprob, s))
        items.append(DiffusionSIRItem(s, float(r), tgt, w.raw_log_importance_ratio, w.applied_log_importance_ratio,
                                      w.log_weight))
    lw = [it.log_weight for it in items]
    probs = normalize_log_weights(lw)
    return DiffusionSIRResult(tuple(items), probs, int(rng.choice(len(items), p=probs)),
                              importance_effective_sample_size(lw))


@dataclass(frozen=True, slots=True)
class DiffusionRolloutEvaluation:
    token_ids: TokenSequence
    reward: float
    proposal_trajectory_logprob: float | None
    target_trajectory_logprob: float | None
    raw_log_importance_ratio: float | None
    applied_log_importance_ratio: float | None
    log_weight: float
    proposal_model_id: str
    proposal_policy_id: str


@dataclass(frozen=True, slots=True)
class DiffusionConditionalCandidate:
    token_ids: TokenSequence
    rollouts: tuple[DiffusionRolloutEvaluation, ...]
    log_weight: float


@dataclass(frozen=True, slots=True)
class DiffusionConditionalISStep:
    generated_length_before: int
    candidates: tuple[DiffusionConditionalCandidate, ...]
    probabilities: tuple[float, ...]
    selected_index: int

    @property
    def selected(self) -> DiffusionConditionalCandidate:
        return self.candidates[self.selected_index]


@dataclass(frozen=True, slots=True)
class DiffusionConditionalISResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[DiffusionConditionalISStep, ...]


def evaluate_rewards(prompt: TokenSequence, continuations: Sequence[TokenSequence],
                     reward: DiffusionRewardFunction | None, reward_batch: DiffusionRewardBatchFunction | None
                     ) -> list[float]:
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one of reward or reward_batch")
    vals = list(reward_batch(prompt, continuations)) if reward_batch is not None else [
        reward(prompt, c) for c in continuations]
    if len(vals) != len(continuations):
        raise RuntimeError("reward evaluator returned an invalid number of values")
    return [float(v) for v in vals]


class DiffusionStepwiseAdapter:
    """Conditional diffusion generation exposed through the shared stepwise protocol."""

    def __init__(self, *, base_backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                 base_sampling: DiffusionSamplingConfig, reward, rollout_backend: DiffusionBackend,
                 rollout_sampling: DiffusionSamplingConfig, target_rollout_backend: DiffusionBackend,
                 target_rollout_sampling: DiffusionSamplingConfig, apply_importance_correction: bool,
                 reward_batch=None):
        self.base_backend, self.prompt, self.config = base_backend, prompt, config
        self.base_sampling, self.reward, self.reward_batch = base_sampling, reward, reward_batch
        self.rollout_backend, self.rollout_sampling = rollout_backend, rollout_sampling
        self.target_backend, self.target_sampling = target_rollout_backend, target_rollout_sampling
        self.stage_lengths = diffusion_decision_stage_lengths(prompt_length=len(prompt),
                                                              total_length=config.total_length,
                                                              decision_block_size=config.block_size,
                                                              sampling=base_sampling)
        self.same_policy = (rollout_backend.model_id == target_rollout_backend.model_id
                            and rollout_sampling.policy_id == target_rollout_sampling.policy_id)
        self.needs_correction = apply_importance_correction and not self.same_policy
        if self.needs_correction:
            if not rollout_sampling.has_exact_trajectory_density:
                raise ValueError("off-policy dLLM IS requires random remasking and positive temperature")
            if not target_rollout_sampling.has_exact_trajectory_density:
                raise ValueError("the target dLLM policy must define an exact trajectory density")
            if (rollout_sampling.block_length, rollout_sampling.steps_per_block) != (
                    target_rollout_sampling.block_length, target_rollout_sampling.steps_per_block):
                raise ValueError("proposal and target trajectory schedules must match")

    initial_state: TokenSequence = ()

    def is_terminal(self, state: TokenSequence) -> bool:
        return len(state) >= self.config.total_length

    def propose(self, state, step_index, seeds: SeedStream):
        n = self.stage_lengths[step_index]
        reqs = [DiffusionGenerationRequest(self.prompt + state, n, self.base_sampling,
                                           seeds.derive("dllm-is", step_index, "candidate", c),
                                           f"dllm-is:step:{step_index}:candidate:{c}")
                for c in range(self.config.candidate_count)]
        out = self.base_backend.sample_batch(reqs)
        if len(out) != self.config.candidate_count:
            raise RuntimeError("backend returned an invalid number of dLLM candidates")
        return out

    def evaluate(self, state, proposals, step_index, seeds: SeedStream):
        cfg = self.config
        remaining = cfg.total_length - len(state) - self.stage_lengths[step_index]
        obs: list[list[RolloutObservation]] = [[] for _ in proposals]
        if remaining == 0:
            rewards = evaluate_rewards(self.prompt, [state + p.token_ids for p in proposals], self.reward,
                                       self.reward_batch)
            for c, r in enumerate(rewards):
                obs[c].append(RolloutObservation(r, 0.0, 0.0, ((), self.base_backend.model_id,
                                                                  self.base_sampling.policy_id)))
            provider = MonteCarloRolloutWeightProvider(reward_temperature=cfg.reward_temperature,
                                                       correction="identity")
        else:
            reqs, owners = [], []
            for c, cand in enumerate(proposals):
                for r in range(cfg.rollout_count):
                    reqs.append(DiffusionGenerationRequest(
                        self.prompt + state + cand.token_ids, remaining, self.rollout_sampling,
                        seeds.derive("dllm-is", step_index, "rollout", c, r),
                        f"dllm-is:step:{step_index}:candidate:{c}:rollout:{r}"))
                    owners.append(c)
            samples = self.rollout_backend.sample_batch(reqs)
            if len(samples) != len(reqs):
                raise RuntimeError("backend returned an invalid number of dLLM rollouts")
            targets = None
            if self.needs_correction:
                targets = self.target_backend.score_trajectories(
                    [DiffusionTrajectoryScoreRequest(s, self.target_sampling) for s in samples])
                if len(targets) != len(samples):
                    raise RuntimeError("backend returned an invalid number of trajectory scores")
            rewards = evaluate_rewards(self.prompt, [state + proposals[o].token_ids + s.token_ids
                                                     for o, s in zip(owners, samples)], self.reward,
                                       self.reward_batch)
            for i, (o, s, r) in enumerate(zip(owners, samples, rewards)):
                if self.needs_correction and s.trajectory_logprob is None:
                    raise RuntimeError("proposal omitted an exact trajectory score")
                obs[o].append(RolloutObservation(r, float(targets[i]) if targets is not None else None,
                                                 s.trajectory_logprob, (s.token_ids, s.model_id, s.policy_id)))
            mode = "importance" if self.needs_correction else ("identity" if self.same_policy else "none")
            provider = MonteCarloRolloutWeightProvider(
                reward_temperature=cfg.reward_temperature, correction=mode,
                log_ratio_clip=cfg.importance_log_ratio_clip if mode == "importance" else None)
        out = []
        for cand, o in zip(proposals, obs):
            est = provider.estimate(o)
            rolls = tuple(DiffusionRolloutEvaluation(
                w.observation.payload[0], w.observation.reward, w.observation.proposal_logprob,
                w.observation.target_logprob, w.raw_log_importance_ratio, w.applied_log_importance_ratio,
                w.log_weight, w.observation.payload[1], w.observation.payload[2]) for w in est.rollouts)
            out.append(StepwiseCandidate(DiffusionConditionalCandidate(cand.token_ids, rolls, est.log_weight),
                                         est.log_weight))
        return tuple(out)

    def advance(self, state, selected: DiffusionConditionalCandidate, step_index):
        return state + selected.token_ids


def run_conditional_diffusion_is(*, base_backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                                 base_sampling: DiffusionSamplingConfig, reward=None, seed: int = 0,
                                 rollout_backend: DiffusionBackend | None = None,
                                 rollout_sampling: DiffusionSamplingConfig | None = None,
                                 target_rollout_backend: DiffusionBackend | None = None,
                                 target_rollout_sampling: DiffusionSamplingConfig | None = None,
                                 apply_importance_correction: bool = True, reward_batch=None
                                 ) -> DiffusionConditionalISResult:
    """Blockwise conditional IS with complete dLLM rollouts (see the module docstring)."""
    adapter = DiffusionStepwiseAdapter(
        base_backend=base_backend, prompt=prompt, config=config, base_sampling=base_sampling, reward=reward,
        rollout_backend=rollout_backend or base_backend, rollout_sampling=rollout_sampling or base_sampling,
        target_rollout_backend=target_rollout_backend or base_backend,
        target_rollout_sampling=target_rollout_sampling or base_sampling,
        apply_importance_correction=apply_importance_correction, reward_batch=reward_batch)
    res = run_stepwise_generation(adapter, SeedStream(seed), selection_namespace=("dllm-is",))
    steps = tuple(DiffusionConditionalISStep(len(s.state_before), tuple(c.value for c in s.candidates),
                                             s.probabilities, s.selected_index) for s in res.steps)
    return DiffusionConditionalISResult(prompt, res.final_state, steps)


__all__ = ["DiffusionConditionalCandidate", "DiffusionConditionalISResult", "DiffusionConditionalISStep",
           "DiffusionRewardBatchFunction", "DiffusionRewardFunction", "DiffusionRolloutEvaluation",
           "DiffusionSIRItem", "DiffusionSIRResult", "DiffusionStepwiseAdapter", "evaluate_rewards",
           "resample_diffusion_candidates", "run_conditional_diffusion_is"]
