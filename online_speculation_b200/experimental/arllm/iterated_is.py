"""Iterated SIR over conditional-IS blocks with a finite pool.

The extended state of a block is a base candidate together with every rollout its
conditional weight was estimated from.  All 1 + U (N - 1) states a block can use
are drawn and weighted up front in one batched backend call; the U i-SIR
transitions then only reshuffle those evaluated states: each pool is the current
state (with its original estimate, never re-estimated) plus the next N - 1 fresh
ones.  The reward has to be a fixed pointwise function of the completed sequence;
a batch-normalised or history-dependent reward would change the target during the
chain.  Stream names follow src/inference_scaling/experimental/arllm/iterated_is.py.
"""

from __future__ import annotations

from dataclasses import dataclass

from ...arllm.algorithms.conditional_is import (ConditionalCandidate, TokenBatchReward, TokenReward,
                                                 _check_policies, estimate_conditional_weights, sample_candidates)
from ...arllm.config import IteratedConditionalISConfig, SamplingConfig
from ...arllm.types import AutoregressiveBackend
from ...shared.rng import SeedStream
from ...shared.stepwise import StepwiseCandidate
from ...shared.types import TokenSequence
from ..shared.iterated_sir import IteratedSIRTransition, iterated_sir_transition


@dataclass(frozen=True, slots=True)
class IteratedConditionalISStep:
    generated_length_before: int
    evaluated_candidates: tuple[ConditionalCandidate, ...]
    transitions: tuple[IteratedSIRTransition[ConditionalCandidate], ...]

    def __post_init__(self) -> None:
        if not self.evaluated_candidates or not self.transitions:
            raise ValueError("an iterated conditional-IS step needs candidates and transitions")

    @property
    def candidates(self) -> tuple[ConditionalCandidate, ...]:
        return self.evaluated_candidates

    @property
    def selected(self) -> ConditionalCandidate:
        return self.transitions[-1].selected.value

    @property
    def selected_index(self) -> int:
        """Position of the selected state among the evaluated states (identity, not equality)."""
        chosen = self.selected
        return next(i for i, c in enumerate(self.evaluated_candidates) if c is chosen)

    @property
    def retained_previous_updates(self) -> int:
        return sum(t.retained_previous for t in self.transitions)


@dataclass(frozen=True, slots=True)
class IteratedConditionalISResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[IteratedConditionalISStep, ...]

    @property
    def fresh_candidate_evaluations(self) -> int:
        return sum(len(s.evaluated_candidates) for s in self.steps)

    @property
    def reused_pool_entries(self) -> int:
        return sum(len(s.transitions) for s in self.steps)


def _pools(evaluated, updates: int, fresh_per_pool: int):
    """The fresh states of every transition, in draw order after the initial state."""
    need = 1 + updates * fresh_per_pool
    if len(evaluated) != need:
        raise RuntimeError(f"{len(evaluated)} evaluated states for {updates} pools of {fresh_per_pool} fresh ones")
    rest = evaluated[1:]
    return [rest[u * fresh_per_pool:(u + 1) * fresh_per_pool] for u in range(updates)]


def iterated_conditional_is_step(*, base_backend: AutoregressiveBackend, rollout_backend: AutoregressiveBackend,
                                 prompt: TokenSequence, generated_prefix: TokenSequence,
                                 config: IteratedConditionalISConfig, base_sampling: SamplingConfig,
                                 rollout_sampling: SamplingConfig, reward: TokenReward | None, seeds: SeedStream,
                                 step_index: int, reward_batch: TokenBatchReward | None = None
                                 ) -> IteratedConditionalISStep:
    _check_policies(base_sampling, rollout_sampling)
    prompt, generated_prefix = tuple(prompt), tuple(generated_prefix)
    remaining = config.total_length - len(generated_prefix)
    if remaining <= 0:
        raise ValueError("the generated prefix already has total_length tokens")
    block = min(config.block_size, remaining)
    drawn = sample_candidates(base_backend, prompt + generated_prefix, config.fresh_candidate_evaluations, block,
                              base_sampling, seeds, step_index)
    evaluated = estimate_conditional_weights(
        base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt, generated_prefix=generated_prefix,
        candidates=drawn, rollout_length=max(0, remaining - block), rollout_count=config.rollout_count,
        base_sampling=base_sampling, rollout_sampling=rollout_sampling, reward_temperature=config.reward_temperature,
        importance_log_ratio_clip=config.importance_log_ratio_clip,
        apply_importance_correction=config.apply_importance_correction, reward=reward, seeds=seeds,
        step_index=step_index, reward_batch=reward_batch)
    state = StepwiseCandidate(evaluated[0], evaluated[0].log_weight)
    transitions = []
    for u, fresh in enumerate(_pools(evaluated, config.updates, config.pool_size - 1)):
        move = iterated_sir_transition(state, [StepwiseCandidate(c, c.log_weight) for c in fresh],
                                       rng=seeds.generator("iterated_conditional_is", step_index, u, "select"))
        transitions.append(move)
        state = move.selected
    return IteratedConditionalISStep(len(generated_prefix), evaluated, tuple(transitions))


def run_iterated_conditional_is(base_backend: AutoregressiveBackend, prompt: TokenSequence,
                                config: IteratedConditionalISConfig, reward: TokenReward | None,
                                seeds: SeedStream, *, base_sampling: SamplingConfig | None = None,
                                rollout_backend: AutoregressiveBackend | None = None,
                                rollout_sampling: SamplingConfig | None = None,
                                reward_batch: TokenBatchReward | None = None) -> IteratedConditionalISResult:
    base_sampling = base_sampling if base_sampling is not None else SamplingConfig()
    rollout_sampling = rollout_sampling if rollout_sampling is not None else base_sampling
    rollout_backend = rollout_backend if rollout_backend is not None else base_backend
    _check_policies(base_sampling, rollout_sampling)
    prompt = tuple(prompt)
    eos = base_sampling.eos_token_id
    text: tuple = ()
    steps: list[IteratedConditionalISStep] = []

    def finished() -> bool:
        return len(text) >= config.total_length or (eos is not None and eos in text)

    while not finished():
        step = iterated_conditional_is_step(base_backend=base_backend, rollout_backend=rollout_backend,
                                            prompt=prompt, generated_prefix=text, config=config,
                                            base_sampling=base_sampling, rollout_sampling=rollout_sampling,
                                            reward=reward, seeds=seeds, step_index=len(steps),
                                            reward_batch=reward_batch)
        steps.append(step)
        text += tuple(step.selected.token_ids)
        if eos is not None and eos in text:
            text = text[:text.index(eos) + 1]
    return IteratedConditionalISResult(prompt, text, tuple(steps))


__all__ = ["IteratedConditionalISResult", "IteratedConditionalISStep", "iterated_conditional_is_step",
           "run_iterated_conditional_is"]
