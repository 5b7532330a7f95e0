"""Finite-pool iterated SIR for conditional autoregressive generation.

The extended state of one block is a base candidate together with every
rollout used to estimate its conditional weight.  All 1 + U (N - 1) fresh
states of a block are sampled and weighted in ONE batched backend call; then U
i-SIR transitions run over them, each keeping the current state (with its
original rollout estimate, not a re-estimate) in slot 0 of a pool of N.  The
reward must be a fixed pointwise function of the completed sequence: a
batch-normalised or history-dependent reward changes the target during the
chain and breaks the invariance argument.

Reference behaviour: src/inference_scaling/experimental/arllm/iterated_is.py:32-226.
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


def iterated_conditional_is_step(*, base_backend: AutoregressiveBackend, rollout_backend: AutoregressiveBackend,
                                 prompt: TokenSequence, generated_prefix: TokenSequence,
                                 config: IteratedConditionalISConfig, base_sampling: SamplingConfig,
                                 rollout_sampling: SamplingConfig, reward: TokenReward | None, seeds: SeedStream,
                                 step_index: int, reward_batch: TokenBatchReward | None = None
                                 ) -> IteratedConditionalISStep:
    _check_policies(base_sampling, rollout_sampling)
    prompt, generated_prefix = tuple(prompt), tuple(generated_prefix)
    left = config.total_length - len(generated_prefix)
    if left <= 0:
        raise ValueError("generated prefix has already reached total_length")
    block = min(config.block_size, left)
    cands = sample_candidates(base_backend, prompt + generated_prefix, config.fresh_candidate_evaluations, block,
                              base_sampling, seeds, step_index)
    evaluated = estimate_conditional_weights(
        base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt, generated_prefix=generated_prefix,
        candidates=cands, rollout_length=max(0, left - block), rollout_count=config.rollout_count,
        base_sampling=base_sampling, rollout_sampling=rollout_sampling, reward_temperature=config.reward_temperature,
        importance_log_ratio_clip=config.importance_log_ratio_clip,
        apply_importance_correction=config.apply_importance_correction, reward=reward, seeds=seeds,
        step_index=step_index, reward_batch=reward_batch)
    current = StepwiseCandidate(evaluated[0], evaluated[0].log_weight)
    fresh_per = config.pool_size - 1
    transitions = []
    for u in range(config.updates):
        group = evaluated[1 + u * fresh_per: 1 + (u + 1) * fresh_per]
        if len(group) != fresh_per:
            raise RuntimeError("candidate grouping does not match the i-SIR configuration")
        t = iterated_sir_transition(current, [StepwiseCandidate(c, c.log_weight) for c in group],
                                    rng=seeds.generator("iterated_conditional_is", step_index, u, "select"))
        transitions.append(t)
        current = t.selected
    return IteratedConditionalISStep(len(generated_prefix), evaluated, tuple(transitions))


def run_iterated_conditional_is(base_backend: AutoregressiveBackend, prompt: TokenSequence,
                                config: IteratedConditionalISConfig, reward: TokenReward | None,
                                seeds: SeedStream, *, base_sampling: SamplingConfig | None = None,
                                rollout_backend: AutoregressiveBackend | None = None,
                                rollout_sampling: SamplingConfig | None = None,
                                reward_batch: TokenBatchReward | None = None) -> IteratedConditionalISResult:
    base_sampling = base_sampling or SamplingConfig()
    rollout_sampling = rollout_sampling or base_sampling
    rollout_backend = rollout_backend or base_backend
    _check_policies(base_sampling, rollout_sampling)
    prompt = tuple(prompt)
    eos = base_sampling.eos_token_id
    gen: TokenSequence = ()
    steps = []
    while len(gen) < config.total_length and (eos is None or eos not in gen):
        st = iterated_conditional_is_step(base_backend=base_backend, rollout_backend=rollout_backend, prompt=prompt,
                                          generated_prefix=gen, config=config, base_sampling=base_sampling,
                                          rollout_sampling=rollout_sampling, reward=reward, seeds=seeds,
                                          step_index=len(steps), reward_batch=reward_batch)
        gen += st.selected.token_ids
        if eos is not None and eos in gen:
            gen = gen[:gen.index(eos) + 1]
        steps.append(st)
    return IteratedConditionalISResult(prompt, gen, tuple(steps))


__all__ = ["IteratedConditionalISResult", "IteratedConditionalISStep", "iterated_conditional_is_step",
           "run_iterated_conditional_is"]
