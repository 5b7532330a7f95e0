"""Method registry: names, report components and runnable entry points.

``METHOD_SPECS`` keeps the reference's method names and the report components
each belongs to (quality, pass@k, distribution, async, dynamic IS, ...), so
suites select the same method sets.  ``run_ar_method`` maps an autoregressive
method name to this package's sampler and returns the completion plus the
method's own diagnostics, for any backend implementing the autoregressive
contract (the sm_100a engine backend or the CPU tabular oracle).

Reference behaviour: experiments/shared/methods.py:8-222 (names and
components); the per-method dispatch of experiments/arllm/gsm8k_reproduction.py
:589-1075.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass, field

from ..arllm.algorithms.conditional_is import run_conditional_is
from ..arllm.algorithms.mh import run_mh_chains_batched, run_reward_mh_chain
from ..arllm.config import (ConditionalISConfig, IteratedConditionalISConfig, MHConfig, ProgressiveISConfig,
                            RewardMHConfig, SamplingConfig, SMCForestConfig)
from ..arllm.types import AutoregressiveBackend, GenerationRequest
from ..shared.rng import SeedStream
from ..shared.types import TokenSequence


@dataclass(frozen=True, slots=True)
class MethodSpec:
    family: str
    name: str
    components: frozenset[str]
    requires_proposal: bool = False
    requires_adapter: bool = False
    paired: bool = True


def _spec(family, name, *components, requires_proposal=False, requires_adapter=False, paired=True) -> MethodSpec:
    return MethodSpec(family, name, frozenset(components), requires_proposal, requires_adapter, paired)


METHOD_SPECS = (
    _spec("arllm", "base", "quality", "default_quality", "passk", "distribution", "async"),
    _spec("arllm", "beam", "quality", "default_quality"),
    _spec("arllm", "best_of_n", "quality", "default_quality", "async"),
    _spec("arllm", "mh", "quality", "default_quality", "passk"),
    _spec("arllm", "reward_mh", "quality", paired=False),
    _spec("arllm", "conditional_is", "quality", "default_quality", "is_passk", "async"),
    _spec("arllm", "iterated_conditional_is", "quality", paired=False),
    _spec("arllm", "conditional_is_small_proposal", "quality", "default_quality", "is_passk", "async",
          requires_proposal=True),
    _spec("arllm", "conditional_is_small_proposal_unclipped", "is_passk", requires_proposal=True),
    _spec("arllm", "conditional_is_small_proposal_uncorrected", "is_passk", requires_proposal=True),
    _spec("arllm", "verifier_mh", "quality", "matched_target", "distribution"),
    _spec("arllm", "verifier_conditional_is", "quality", "matched_target", "distribution"),
    _spec("arllm", "verifier_conditional_is_small_proposal", "quality", "matched_target", "distribution",
          requires_proposal=True),
    _spec("arllm", "rl_sample", "quality", "default_quality", "passk", "distribution", requires_adapter=True),
    _spec("arllm", "rl_greedy", "quality", "default_quality", requires_adapter=True),
    _spec("arllm", "base_candidate_fixed", "dynamic_is"),
    _spec("arllm", "replay_aware_fixed", "dynamic_is"),
    _spec("arllm", "replay_aware_optimal", "dynamic_is"),
    _spec("arllm", "progressive_is", "experimental", paired=False),
    _spec("arllm", "smc_forest", "experimental", paired=False),
    _spec("dllm", "base", "quality", "default_quality", "passk", "distribution", "async"),
    _spec("dllm", "block_beam", "quality", "default_quality"),
    _spec("dllm", "best_of_n", "quality", "default_quality", "async"),
    _spec("dllm", "trajectory_power_mh", "quality", "default_quality", "passk"),
    _spec("dllm", "conditional_is", "quality", "default_quality", "is_passk", "async"),
    _spec("dllm", "conditional_is_reduced_layer_proposal", "quality", "default_quality", "is_passk", "async",
          requires_proposal=True),
    _spec("dllm", "conditional_is_reduced_layer_proposal_unclipped", "is_passk", "default_quality",
          requires_proposal=True),
    _spec("dllm", "conditional_is_reduced_layer_proposal_uncorrected", "is_passk", "default_quality",
          requires_proposal=True),
    _spec("dllm", "verifier_mh", "quality", "default_quality", "matched_target", "distribution"),
    _spec("dllm", "verifier_conditional_is", "quality", "default_quality", "matched_target", "distribution"),
    _spec("dllm", "verifier_conditional_is_reduced_layer_proposal", "quality", "default_quality", "matched_target",
          "distribution", requires_proposal=True),
    _spec("dllm", "vrpo_sample", "quality", "aligned", "passk", "distribution", requires_adapter=True),
    _spec("dllm", "vrpo_greedy", "quality", "aligned", requires_adapter=True),
    _spec("dllm", "base_candidate_fixed", "dynamic_is"),
    _spec("dllm", "trajectory_replay_aware_fixed", "dynamic_is"),
    _spec("dllm", "trajectory_replay_aware_optimal", "dynamic_is"),
)

METHOD_REGISTRY = {(s.family, s.name): s for s in METHOD_SPECS}
if len(METHOD_REGISTRY) != len(METHOD_SPECS):
    raise RuntimeError("duplicate method specification")


def methods_for(family: str, component: str) -> tuple[str, ...]:
    if family not in ("arllm", "dllm"):
        raise ValueError(f"unknown model family {family!r}")
    return tuple(s.name for s in METHOD_SPECS if s.family == family and component in s.components)


def method_spec(family: str, name: str) -> MethodSpec:
    try:
        return METHOD_REGISTRY[(family, name)]
    except KeyError:
        raise ValueError(f"unknown {family} method {name!r}") from None


AR_METHODS = methods_for("arllm", "quality")
AR_DEFAULT_METHODS = methods_for("arllm", "default_quality")
AR_PASSK_METHODS = methods_for("arllm", "passk")
AR_IS_PASSK_METHODS = methods_for("arllm", "is_passk")
AR_ASYNC_METHODS = methods_for("arllm", "async")
AR_DISTRIBUTION_METHODS = methods_for("arllm", "distribution")
AR_DYNAMIC_METHODS = methods_for("arllm", "dynamic_is")
AR_PAIRED_METHODS = tuple(s.name for s in METHOD_SPECS if s.family == "arllm" and "quality" in s.components
                          and s.paired)
DLLM_METHODS = tuple(s.name for s in METHOD_SPECS if s.family == "dllm")
DLLM_DEFAULT_METHODS = methods_for("dllm", "default_quality")
DLLM_ALIGNED_METHODS = methods_for("dllm", "aligned")
DLLM_DYNAMIC_METHODS = methods_for("dllm", "dynamic_is")


# ------------------------------------------------------------- runnables --
Reward = Callable[[TokenSequence, TokenSequence], float]


@dataclass
class MethodSettings:
    """Budget and policy knobs shared by the runnable AR methods."""

    max_new_tokens: int = 64
    block_size: int = 16
    temperature: float = 1.0
    alpha: float = 4.0
    mh_steps_per_block: int = 4
    reward_temperature: float = 0.5
    candidates: int = 4
    rollouts: int = 4
    best_of: int = 4
    pool_size: int = 3
    updates: int = 2
    particles: int = 4
    eos_token_id: int | None = None
    extra: dict = field(default_factory=dict)


@dataclass(frozen=True, slots=True)
class MethodOutcome:
    method: str
    token_ids: TokenSequence
    diagnostics: dict


def _base_sampling(s: MethodSettings) -> SamplingConfig:
    return SamplingConfig(temperature=s.temperature, eos_token_id=s.eos_token_id)


def run_ar_method(name: str, backend: AutoregressiveBackend, prompt: Sequence[int], settings: MethodSettings,
                  seed: int, *, reward: Reward | None = None) -> MethodOutcome:
    """Run one autoregressive method on one prompt; ``reward`` is required by the reward-tilted methods."""
    method_spec("arllm", name)
    prompt = tuple(prompt)
    s = settings
    seeds = SeedStream(seed)
    if name == "base":
        out = backend.sample_batch([GenerationRequest(prompt, s.max_new_tokens, _base_sampling(s), seed, "base")])[0]
        return MethodOutcome(name, out.token_ids, {"logprob": out.logprob, "finish_reason": out.finish_reason})
    if name == "best_of_n":
        if reward is None:
            raise ValueError("best_of_n needs a reward")
        outs = backend.sample_batch([GenerationRequest(prompt, s.max_new_tokens, _base_sampling(s),
                                                       seeds.derive("best_of_n", i), f"best-of-n:{i}")
                                     for i in range(s.best_of)])
        scores = [float(reward(prompt, o.token_ids)) for o in outs]
        i = max(range(len(outs)), key=lambda j: (scores[j], -j))
        return MethodOutcome(name, outs[i].token_ids, {"rewards": scores, "selected": i})
    if name == "mh":
        cfg = MHConfig(alpha=s.alpha, total_length=s.max_new_tokens, block_size=min(s.block_size, s.max_new_tokens),
                       steps_per_block=s.mh_steps_per_block)
        prop = SamplingConfig(temperature=1.0 / s.alpha)
        res = run_mh_chains_batched(backend, prompt, cfg, prop, [seeds])[0]
        return MethodOutcome(name, res.token_ids, {"acceptance_rate": res.acceptance_rate,
                                                   "attempts": res.attempts})
    if reward is None:
        raise ValueError(f"{name} needs a reward")
    if name in ("reward_mh", "verifier_mh"):
        cfg = RewardMHConfig(total_length=s.max_new_tokens, block_size=min(s.block_size, s.max_new_tokens),
                             steps_per_block=s.mh_steps_per_block, reward_temperature=s.reward_temperature)
        res = run_reward_mh_chain(backend, prompt, cfg, SamplingConfig(), reward, seeds)
        return MethodOutcome(name, res.token_ids, {"reward": res.reward, "acceptance_rate": res.acceptance_rate})
    if name in ("conditional_is", "verifier_conditional_is"):
        cfg = ConditionalISConfig(candidate_count=s.candidates, rollout_count=s.rollouts,
                                  block_size=min(s.block_size, s.max_new_tokens), total_length=s.max_new_tokens,
                                  reward_temperature=s.reward_temperature)
        res = run_conditional_is(backend, prompt, cfg, reward, seeds, base_sampling=_base_sampling(s))
        return MethodOutcome(name, res.token_ids, {"steps": len(res.steps)})
    if name == "iterated_conditional_is":
        from ..experimental.arllm.iterated_is import run_iterated_conditional_is

        cfg = IteratedConditionalISConfig(pool_size=s.pool_size, updates=s.updates, rollout_count=s.rollouts,
                                          block_size=min(s.block_size, s.max_new_tokens),
                                          total_length=s.max_new_tokens, reward_temperature=s.reward_temperature)
        res = run_iterated_conditional_is(backend, prompt, cfg, reward, seeds, base_sampling=_base_sampling(s))
        return MethodOutcome(name, res.token_ids, {"fresh_candidate_evaluations": res.fresh_candidate_evaluations})
    if name == "progressive_is":
        from ..experimental.arllm.progressive_is import run_progressive_conditional_is

        cfg = ProgressiveISConfig(candidate_count=s.candidates, block_size=min(s.block_size, s.max_new_tokens),
                                  total_length=s.max_new_tokens, reward_temperature=s.reward_temperature,
                                  evaluation_cost_budget=float(s.candidates * s.rollouts))
        res = run_progressive_conditional_is(backend, prompt, cfg, reward, seeds, base_sampling=_base_sampling(s))
        return MethodOutcome(name, res.token_ids, {"steps": len(res.steps)})
    if name == "smc_forest":
        from ..experimental.arllm.smc_forest import run_smc_rollout_forest

        cfg = SMCForestConfig(particle_count=s.particles, rollout_count=s.rollouts,
                              block_size=min(s.block_size, s.max_new_tokens), total_length=s.max_new_tokens,
                              reward_temperature=s.reward_temperature)
        res = run_smc_rollout_forest(backend, prompt, cfg, reward, seeds, base_sampling=_base_sampling(s))
        return MethodOutcome(name, res.token_ids, {"reused_rollouts": res.reused_rollouts,
                                                   "fresh_rollouts": res.fresh_rollouts})
    if name in ("base_candidate_fixed", "replay_aware_fixed", "replay_aware_optimal"):
        from ..experimental.arllm.dynamic_is import run_dynamic_is_arm

        res = run_dynamic_is_arm(backend, prompt, arm=name, candidate_count=s.candidates,
                                 block_size=min(s.block_size, s.max_new_tokens), total_length=s.max_new_tokens,
                                 reward=reward, seeds=seeds, reward_temperature=s.reward_temperature,
                                 history=int(s.extra.get("history", 4)),
                                 rollout_budget=float(s.extra.get("rollout_budget", s.candidates * s.rollouts)),
                                 base_sampling=_base_sampling(s))
        est = [c.estimate for st in res.steps for c in st.candidates]
        return MethodOutcome(name, res.token_ids, {"steps": len(res.steps),
                                                   "history_rollouts_reused": sum(e.history_count for e in est),
                                                   "fresh_rollouts": sum(e.fresh_count for e in est)})
    raise NotImplementedError(f"method {name!r} needs resources this runner does not build (a proposal model, "
                              "an adapter or a replay store); call its sampler directly")


RUNNABLE_AR_METHODS = ("base", "best_of_n", "mh", "reward_mh", "verifier_mh", "conditional_is",
                       "verifier_conditional_is", "iterated_conditional_is", "progressive_is", "smc_forest",
                       "base_candidate_fixed", "replay_aware_fixed", "replay_aware_optimal")


__all__ = ["AR_ASYNC_METHODS", "AR_DEFAULT_METHODS", "AR_DISTRIBUTION_METHODS", "AR_DYNAMIC_METHODS",
           "AR_IS_PASSK_METHODS", "AR_METHODS", "AR_PAIRED_METHODS", "AR_PASSK_METHODS", "DLLM_ALIGNED_METHODS",
           "DLLM_DEFAULT_METHODS", "DLLM_DYNAMIC_METHODS", "DLLM_METHODS", "METHOD_REGISTRY", "METHOD_SPECS",
           "MethodOutcome", "MethodSettings", "MethodSpec", "RUNNABLE_AR_METHODS", "method_spec", "methods_for",
           "run_ar_method"]
