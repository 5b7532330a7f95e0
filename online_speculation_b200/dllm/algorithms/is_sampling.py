"""Reward reweighting (SIR) and blockwise conditional importance sampling for masked dLLMs.

Conditional IS commits one decision block at a time.  ``candidate_count`` base
candidates are drawn for the block; each is completed by ``rollout_count`` full
rollouts laid out as one (candidate x rollout) grid and generated in one batch; a
candidate's log weight is the log-mean-exp over its row of r / tau, plus the
trajectory log ratio log p_target(trace) - log q(trace) when the rollouts come from
another model or transition policy; one candidate is then drawn from the normalised
weights.  Decision blocks never split a native diffusion block.  Random-stream names
and request ids follow src/inference_scaling/dllm/algorithms/is_sampling.py.
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
    """One draw from reward-tilted weights (on-policy, or with trajectory importance ratios)."""
    if not len(samples) or len(samples) != len(rewards):
        raise ValueError("samples and rewards must be non-empty and of equal length")
    if not reward_temperature > 0:
        raise ValueError("reward_temperature has to be positive")
    off_policy = target_trajectory_logprobs is not None
    if off_policy:
        if len(target_trajectory_logprobs) != len(samples):
            raise ValueError("off-policy weights need one target trajectory score per sample")
        if any(s.trajectory_logprob is None for s in samples):
            raise ValueError("off-policy weights need the exact proposal trajectory density of every sample")
    provider = MonteCarloRolloutWeightProvider(reward_temperature=reward_temperature,
                                               correction="importance" if off_policy else "none",
                                               log_ratio_clip=importance_log_ratio_clip if off_policy else None)
    targets = [None] * len(samples) if not off_policy else [float(t) for t in target_trajectory_logprobs]
    observations = [RolloutObservation(float(r), t, s.trajectory_logprob, s)
                    for s, r, t in zip(samples, rewards, targets)]
    weighted = provider.estimate(observations).rollouts
    items = tuple(DiffusionSIRItem(w.observation.payload, w.observation.reward, t, w.raw_log_importance_ratio,
                                   w.applied_log_importance_ratio, w.log_weight) for w, t in zip(weighted, targets))
    log_weights = [it.log_weight for it in items]
    probabilities = normalize_log_weights(log_weights)
    return DiffusionSIRResult(items, probabilities, int(rng.choice(len(items), p=probabilities)),
                              importance_effective_sample_size(log_weights))


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
        raise ValueError("give either reward or reward_batch")
    values = list(reward_batch(prompt, continuations)) if reward_batch is not None else \
        [reward(prompt, c) for c in continuations]
    if len(values) != len(continuations):
        raise RuntimeError(f"{len(values)} rewards for {len(continuations)} continuations")
    return [float(v) for v in values]


class DiffusionStepwiseAdapter:
    """Blockwise conditional diffusion generation as a backend of the shared stepwise driver."""

    def __init__(self, *, base_backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                 base_sampling: DiffusionSamplingConfig, reward, rollout_backend: DiffusionBackend,
                 rollout_sampling: DiffusionSamplingConfig, target_rollout_backend: DiffusionBackend,
                 target_rollout_sampling: DiffusionSamplingConfig, apply_importance_correction: bool,
                 reward_batch=None):
        self.base_backend = base_backend
        self.prompt = tuple(prompt)
        self.config = config
        self.base_sampling = base_sampling
        self.reward = reward
        self.reward_batch = reward_batch
        self.rollout_backend = rollout_backend
        self.rollout_sampling = rollout_sampling
        self.target_backend = target_rollout_backend
        self.target_sampling = target_rollout_sampling
        self.stage_lengths = diffusion_decision_stage_lengths(prompt_length=len(prompt),
                                                              total_length=config.total_length,
                                                              decision_block_size=config.block_size,
                                                              sampling=base_sampling)
        self.same_policy = (rollout_backend.model_id, rollout_sampling.policy_id) == \
            (target_rollout_backend.model_id, target_rollout_sampling.policy_id)
        self.needs_correction = apply_importance_correction and not self.same_policy
        if self.needs_correction:
            self._check_densities()

    def _check_densities(self) -> None:
        if not self.rollout_sampling.has_exact_trajectory_density:
            raise ValueError("off-policy dLLM weights need random remasking at a positive temperature")
        if not self.target_sampling.has_exact_trajectory_density:
            raise ValueError("the target dLLM policy has no exact trajectory density")
        schedule = lambda s: (s.block_length, s.steps_per_block)   # noqa: E731
        if schedule(self.rollout_sampling) != schedule(self.target_sampling):
            raise ValueError("proposal and target trajectories follow different schedules")

    initial_state: TokenSequence = ()

    def is_terminal(self, state: TokenSequence) -> bool:
        return len(state) >= self.config.total_length

    def propose(self, state, step_index, seeds: SeedStream):
        length = self.stage_lengths[step_index]
        requests = [DiffusionGenerationRequest(self.prompt + tuple(state), length, self.base_sampling,
                                               seeds.derive("dllm-is", step_index, "candidate", c),
                                               f"dllm-is:step:{step_index}:candidate:{c}")
                    for c in range(self.config.candidate_count)]
        drawn = self.base_backend.sample_batch(requests)
        if len(drawn) != len(requests):
            raise RuntimeError(f"{len(drawn)} dLLM candidates came back for {len(requests)}")
        return drawn

    def _terminal_observations(self, state, proposals):
        rewards = evaluate_rewards(self.prompt, [tuple(state) + tuple(p.token_ids) for p in proposals],
                                   self.reward, self.reward_batch)
        tag = ((), self.base_backend.model_id, self.base_sampling.policy_id)
        rows = [[RolloutObservation(r, 0.0, 0.0, tag)] for r in rewards]
        return rows, "identity"

    def _rollout_observations(self, state, proposals, step_index, remaining, seeds):
        cfg = self.config
        grid = [(c, r) for c in range(len(proposals)) for r in range(cfg.rollout_count)]
        requests = [DiffusionGenerationRequest(self.prompt + tuple(state) + tuple(proposals[c].token_ids), remaining,
                                               self.rollout_sampling,
                                               seeds.derive("dllm-is", step_index, "rollout", c, r),
                                               f"dllm-is:step:{step_index}:candidate:{c}:rollout:{r}")
                    for c, r in grid]
        rollouts = self.rollout_backend.sample_batch(requests)
        if len(rollouts) != len(requests):
            raise RuntimeError(f"{len(rollouts)} dLLM rollouts came back for {len(requests)}")
        targets = [None] * len(rollouts)
        if self.needs_correction:
            if any(s.trajectory_logprob is None for s in rollouts):
                raise RuntimeError("a rollout came back without its exact trajectory density")
            scores = self.target_backend.score_trajectories(
                [DiffusionTrajectoryScoreRequest(s, self.target_sampling) for s in rollouts])
            if len(scores) != len(rollouts):
                raise RuntimeError(f"{len(scores)} trajectory scores for {len(rollouts)} rollouts")
            targets = [float(t) for t in scores]
        texts = [tuple(state) + tuple(proposals[c].token_ids) + tuple(s.token_ids) for (c, _), s in zip(grid, rollouts)]
        rewards = evaluate_rewards(self.prompt, texts, self.reward, self.reward_batch)
        rows: list[list[RolloutObservation]] = [[] for _ in proposals]
        for (c, _), s, r, t in zip(grid, rollouts, rewards, targets):
            rows[c].append(RolloutObservation(r, t, s.trajectory_logprob, (s.token_ids, s.model_id, s.policy_id)))
        mode = "importance" if self.needs_correction else ("identity" if self.same_policy else "none")
        return rows, mode

    def evaluate(self, state, proposals, step_index, seeds: SeedStream):
        cfg = self.config
        remaining = cfg.total_length - len(state) - self.stage_lengths[step_index]
        if remaining == 0:
            rows, mode = self._terminal_observations(state, proposals)
        else:
            rows, mode = self._rollout_observations(state, proposals, step_index, remaining, seeds)
        provider = MonteCarloRolloutWeightProvider(
            reward_temperature=cfg.reward_temperature, correction=mode,
            log_ratio_clip=cfg.importance_log_ratio_clip if mode == "importance" else None)
        scored = []
        for proposal, row in zip(proposals, rows):
            estimate = provider.estimate(row)
            evaluations = tuple(DiffusionRolloutEvaluation(
                w.observation.payload[0], w.observation.reward, w.observation.proposal_logprob,
                w.observation.target_logprob, w.raw_log_importance_ratio, w.applied_log_importance_ratio,
                w.log_weight, w.observation.payload[1], w.observation.payload[2]) for w in estimate.rollouts)
            candidate = DiffusionConditionalCandidate(proposal.token_ids, evaluations, estimate.log_weight)
            scored.append(StepwiseCandidate(candidate, estimate.log_weight))
        return tuple(scored)

    def advance(self, state, selected: DiffusionConditionalCandidate, step_index):
        return tuple(state) + tuple(selected.token_ids)


def run_conditional_diffusion_is(*, base_backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionISConfig,
                                 base_sampling: DiffusionSamplingConfig, reward=None, seed: int = 0,
                                 rollout_backend: DiffusionBackend | None = None,
                                 rollout_sampling: DiffusionSamplingConfig | None = None,
                                 target_rollout_backend: DiffusionBackend | None = None,
                                 target_rollout_sampling: DiffusionSamplingConfig | None = None,
                                 apply_importance_correction: bool = True, reward_batch=None
                                 ) -> DiffusionConditionalISResult:
    """Blockwise conditional IS with complete dLLM rollouts."""
    adapter = DiffusionStepwiseAdapter(
        base_backend=base_backend, prompt=prompt, config=config, base_sampling=base_sampling, reward=reward,
        rollout_backend=rollout_backend if rollout_backend is not None else base_backend,
        rollout_sampling=rollout_sampling if rollout_sampling is not None else base_sampling,
        target_rollout_backend=target_rollout_backend if target_rollout_backend is not None else base_backend,
        target_rollout_sampling=target_rollout_sampling if target_rollout_sampling is not None else base_sampling,
        apply_importance_correction=apply_importance_correction, reward_batch=reward_batch)
    run = run_stepwise_generation(adapter, SeedStream(seed), selection_namespace=("dllm-is",))
    steps = tuple(DiffusionConditionalISStep(len(sel.state_before), tuple(c.value for c in sel.candidates),
                                             sel.probabilities, sel.selected_index) for sel in run.steps)
    return DiffusionConditionalISResult(prompt, run.final_state, steps)


__all__ = ["DiffusionConditionalCandidate", "DiffusionConditionalISResult", "DiffusionConditionalISStep",
           "DiffusionRewardBatchFunction", "DiffusionRewardFunction", "DiffusionRolloutEvaluation",
           "DiffusionSIRItem", "DiffusionSIRResult", "DiffusionStepwiseAdapter", "evaluate_rewards",
           "resample_diffusion_candidates", "run_conditional_diffusion_is"]
