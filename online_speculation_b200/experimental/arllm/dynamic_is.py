"""Dynamic candidate proposals with replay-corrected conditional weights.

Three mechanisms on top of base-candidate replay:

* a defensive candidate mixture q = (1 - m) p_base + m p_aux: candidate k uses
  the auxiliary proposal with probability m (explicit uniform per candidate),
  and its exact mixture probability is computed by scoring the block under both
  policies, so the outer weight log p_base - log q is exact;
* a frozen variance-cost allocation of replay history and fresh base rollouts
  per candidate (statistics come from a pluggable provider that sees only the
  design pool and inventory counts, never the evaluation records it will use);
* the completion-level truncated replay estimator of base replay, unchanged.

The candidate weight is outer log ratio + replay log weight, and one candidate
is drawn with the step's selection uniform.

Reference behaviour: src/inference_scaling/experimental/arllm/dynamic_is.py:55-789.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, replace
from math import exp, isfinite, log

import numpy as np

from ...arllm.algorithms.base_replay import (ReplayWeightEstimate, build_fresh_replay_requests,
                                             estimate_replay_weight, write_reserve_records)
from ...arllm.algorithms.conditional_is import TokenReward, _full_support
from ...arllm.config import DynamicISConfig, SamplingConfig
from ...arllm.replay import (BehaviorPolicy, BehaviorRegistry, InMemoryReplayStore, ReplayKey, ReplaySampleRequest,
                             mixture_logprobabilities, sample_replay_records, score_continuations,
                             validate_record_probabilities)
from ...arllm.types import AutoregressiveBackend, GenerationRequest, ScoreRequest
from ...shared.budget import BudgetAllocation, VarianceCostEstimate, allocate_variance_cost_budget
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence


@dataclass(frozen=True, slots=True)
class CandidateProposal:
    proposal_id: str
    backend: AutoregressiveBackend
    sampling: SamplingConfig

    @classmethod
    def for_backend(cls, backend: AutoregressiveBackend, sampling: SamplingConfig, *,
                    label: str | None = None) -> "CandidateProposal":
        return cls(label or f"{backend.model_id}|{sampling.policy_id}", backend, sampling)


@dataclass(frozen=True, slots=True)
class DynamicCandidateDraw:
    token_ids: TokenSequence
    base_token_logprobs: tuple[float, ...]
    base_logprob: float
    auxiliary_logprob: float
    proposal_logprob: float
    outer_log_ratio: float
    source: str
    auxiliary_proposal_id: str | None


CandidateProposalFactory = Callable[[int, int, tuple[DynamicCandidateDraw, ...]], CandidateProposal]
CandidateProposalSource = CandidateProposal | CandidateProposalFactory | None


@dataclass(frozen=True, slots=True)
class DesignStatisticsContext:
    key: ReplayKey
    evaluation_inventory: tuple[tuple[str, int], ...]
    store: InMemoryReplayStore
    registry: BehaviorRegistry
    base_policy: BehaviorPolicy
    reward_temperature: float
    truncation: float

    @property
    def available_history(self) -> int:
        return sum(n for _, n in self.evaluation_inventory)


DesignStatisticsProvider = Callable[[DesignStatisticsContext], VarianceCostEstimate]
DesignPreparation = Callable[[tuple[DesignStatisticsContext, ...]], None]


@dataclass(frozen=True, slots=True)
class RolloutBudgetContext:
    """What a budget provider may see when the step's budget is frozen: the drawn
    candidates and replay inventory counts, never evaluation completions or rewards."""

    draws: tuple[DynamicCandidateDraw, ...]
    keys: tuple[ReplayKey, ...]
    terminal: tuple[bool, ...]
    history_capacities: tuple[int, ...]
    group_capacities: Mapping[ReplayKey, int]


RolloutBudgetProvider = Callable[[RolloutBudgetContext], float]


def constant_design_statistics(context: DesignStatisticsContext) -> VarianceCostEstimate:
    """Cold-start statistics (unit spreads)."""
    return VarianceCostEstimate(history_std=1.0 if context.available_history else 0.0, fresh_std=1.0)


def _sample_std(values: Sequence[float], fallback: float) -> float:
    if len(values) < 2:
        return fallback
    v = float(np.std(np.asarray(values, dtype=np.float64), ddof=1))
    return v if isfinite(v) else fallback


def empirical_design_statistics(context: DesignStatisticsContext) -> VarianceCostEstimate:
    """Spreads and costs estimated from the design pool of the candidate's key only."""
    inv = dict(context.evaluation_inventory)
    design = context.store.design_records(context.key)
    hist = [r for r in design if r.behavior_id in inv]
    base = [r for r in design if r.behavior_id == context.base_policy.behavior_id]
    log_c = log(context.truncation)
    tau = context.reward_temperature
    h_vals: list[float] = []
    if inv and hist:
        validate_record_probabilities(hist, context.registry)
        comps = [r.completion for r in hist]
        p = score_continuations(context.base_policy, context.key, comps)
        b = mixture_logprobabilities(context.registry, context.key, inv, comps)
        h_vals = [exp(min(log_c, lp - lb) + r.reward / tau) for r, lp, lb in zip(hist, p, b)]
    f_vals: list[float] = []
    if base:
        if inv:
            b = mixture_logprobabilities(context.registry, context.key, inv, [r.completion for r in base])
            for r, lb in zip(base, b):
                lr = r.behavior_logprob - lb
                tail = 0.0 if lr <= log_c else 1.0 - exp(log_c - lr)
                f_vals.append(tail * exp(r.reward / tau))
        else:
            f_vals = [exp(r.reward / tau) for r in base]
    mult = 1 + len(inv)   # one base score plus one score per behavior in the mixture

    def cost(rs):
        return max(1.0, mult * sum(len(r.completion) for r in rs) / len(rs)) if rs else 1.0

    return VarianceCostEstimate(history_std=_sample_std(h_vals, 1.0) if context.available_history else 0.0,
                                fresh_std=_sample_std(f_vals, 1.0), history_cost=cost(hist), fresh_cost=cost(base))


@dataclass(frozen=True, slots=True)
class DynamicCandidate:
    draw: DynamicCandidateDraw
    allocation: BudgetAllocation
    estimate: ReplayWeightEstimate
    log_weight: float

    @property
    def token_ids(self) -> TokenSequence:
        return self.draw.token_ids


@dataclass(frozen=True, slots=True)
class DynamicISStep:
    generated_length_before: int
    candidates: tuple[DynamicCandidate, ...]
    selected_index: int

    @property
    def selected(self) -> DynamicCandidate:
        return self.candidates[self.selected_index]


@dataclass(frozen=True, slots=True)
class DynamicISResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    steps: tuple[DynamicISStep, ...]
    reserve_records_written: int


def _score(backend, sampling, prefix, cands: Sequence[TokenSequence]) -> tuple[tuple[float, ...], ...]:
    if not cands:
        return ()
    got = backend.score_batch([ScoreRequest(tuple(prefix), tuple(cands), sampling)])
    if len(got) != len(cands) or any(len(s) != len(c) for s, c in zip(got, cands)):
        raise RuntimeError("candidate proposal returned an invalid score shape")
    return tuple(tuple(s) for s in got)


def _make_draw(sample_tokens, base_scores, aux, aux_scores, used_aux: bool, mixture: float) -> DynamicCandidateDraw:
    lp = float(sum(base_scores))
    if not isfinite(lp):
        raise ValueError("auxiliary candidate proposal generated outside base support")
    la, aux_id = float("-inf"), None
    if aux is not None:
        la, aux_id = float(sum(aux_scores)), aux.proposal_id
        if used_aux and not isfinite(la):
            raise RuntimeError("auxiliary sampler generated a zero-probability candidate")
    lq = lp if mixture == 0 else float(np.logaddexp(log(1.0 - mixture) + lp, log(mixture) + la))
    return DynamicCandidateDraw(tuple(sample_tokens), tuple(base_scores), lp, la, lq, lp - lq,
                                "auxiliary" if used_aux else "base", aux_id)


def draw_candidates(*, base_backend, base_sampling, prefix, count, block, mixture, source, seeds, step):
    """The candidate draws of one dynamic-IS step (the step's own seed stream): a caller that draws them
    first -- to prepare replay history for exactly these blocks -- gets the blocks the step will draw."""
    def component(k):
        return bool(mixture > 0 and seeds.generator("dynamic_is", step, k, "component").random() < mixture)

    def request(k, sampling):
        return GenerationRequest(tuple(prefix), block, sampling, seeds.derive("dynamic_is", step, k, "sample"),
                                 f"dynamic-is:step:{step}:candidate:{k}")

    def check(aux):
        if mixture > 0 and aux is None:
            raise ValueError("a positive auxiliary mixture requires a candidate proposal")
        if aux is not None and aux.sampling.eos_token_id != base_sampling.eos_token_id:
            raise ValueError("base and auxiliary candidate policies must agree on eos_token_id")

    def validate(smp, backend, sampling):
        if not smp.token_ids:
            raise RuntimeError("candidate proposal must return a non-empty candidate")
        if smp.model_id != backend.model_id or smp.policy_id != sampling.policy_id:
            raise RuntimeError("candidate sample does not match its declared proposal")

    if source is None or isinstance(source, CandidateProposal):
        # a fixed proposal: one batched sample call per (backend, policy) and one score call per policy
        aux = source
        check(aux)
        used = [component(k) for k in range(count)]
        groups: dict = {}
        for k, u in enumerate(used):
            be, sp = (aux.backend, aux.sampling) if u else (base_backend, base_sampling)
            groups.setdefault((id(be), sp), (be, sp, []))[2].append(k)
        samples: list = [None] * count
        for be, sp, ks in groups.values():
            got = be.sample_batch([request(k, sp) for k in ks])
            if len(got) != len(ks):
                raise RuntimeError("candidate proposal returned an invalid sample count")
            for k, smp in zip(ks, got):
                validate(smp, be, sp)
                samples[k] = smp
        toks = [tuple(s.token_ids) for s in samples]
        base_sc = _score(base_backend, None, prefix, toks)
        aux_sc = _score(aux.backend, aux.sampling, prefix, toks) if aux is not None else [None] * count
        return tuple(_make_draw(t, b, aux, a, u, mixture) for t, b, a, u in zip(toks, base_sc, aux_sc, used))
    # an adaptive proposal: the factory sees the earlier draws of this step, so candidates go one at a time
    draws: list[DynamicCandidateDraw] = []
    for k in range(count):
        aux = source(step, k, tuple(draws))
        if not isinstance(aux, CandidateProposal):
            raise TypeError("candidate proposal factory must return CandidateProposal")
        check(aux)
        u = component(k)
        be, sp = (aux.backend, aux.sampling) if u else (base_backend, base_sampling)
        got = be.sample_batch([request(k, sp)])
        if len(got) != 1:
            raise RuntimeError("candidate proposal must return one non-empty candidate")
        validate(got[0], be, sp)
        t = tuple(got[0].token_ids)
        draws.append(_make_draw(t, _score(base_backend, None, prefix, [t])[0], aux,
                                _score(aux.backend, aux.sampling, prefix, [t])[0], u, mixture))
    return tuple(draws)


def dynamic_is_step(*, base_backend: AutoregressiveBackend, registry: BehaviorRegistry, store: InMemoryReplayStore,
                    prompt: TokenSequence, generated_prefix: TokenSequence, config: DynamicISConfig,
                    base_sampling: SamplingConfig, reward: TokenReward, reward_version: str, seeds: SeedStream,
                    step_index: int, auxiliary_proposal: CandidateProposalSource = None,
                    statistics_provider: DesignStatisticsProvider = constant_design_statistics,
                    design_prepare: DesignPreparation | None = None,
                    rollout_budget_provider: RolloutBudgetProvider | None = None) -> DynamicISStep:
    _full_support(base_sampling, "base candidates")
    prompt, generated_prefix = tuple(prompt), tuple(generated_prefix)
    left = config.total_length - len(generated_prefix)
    if left <= 0:
        raise ValueError("generated prefix has already reached total_length")
    block = min(config.block_size, left)
    draws = draw_candidates(base_backend=base_backend, base_sampling=base_sampling, prefix=prompt + generated_prefix,
                             count=config.candidate_count, block=block, mixture=config.auxiliary_mixture,
                             source=auxiliary_proposal, seeds=seeds, step=step_index)
    base_policy = BehaviorPolicy.for_backend(base_backend, base_sampling, label="base")
    registry.register(base_policy)
    roll = max(0, left - block)
    eos = base_sampling.eos_token_id
    keys = [ReplayKey(prompt, generated_prefix, d.token_ids, reward_version) for d in draws]
    terminal = [roll == 0 or (eos is not None and d.token_ids[-1] == eos) for d in draws]
    inv = {k: store.inventory(k) for k in dict.fromkeys(keys)}
    group_caps = {k: sum(v.values()) for k, v in inv.items()}
    contexts: list[DesignStatisticsContext | None] = []
    hist_caps, min_fresh = [], []
    for key, term in zip(keys, terminal):
        if term:
            contexts.append(None)
            hist_caps.append(0)
            min_fresh.append(0)
            continue
        ctx = DesignStatisticsContext(key, tuple(sorted(inv[key].items())), store, registry, base_policy,
                                      config.reward_temperature, config.truncation)
        contexts.append(ctx)
        hist_caps.append(min(config.max_history_per_candidate, ctx.available_history))
        min_fresh.append(config.minimum_fresh_per_candidate)
    if design_prepare is not None:
        design_prepare(tuple(c for c in contexts if c is not None))
    stats = [VarianceCostEstimate(0.0, 0.0) if c is None else statistics_provider(c) for c in contexts]
    outer = np.asarray([d.outer_log_ratio for d in draws], dtype=np.float64)
    # a common scale cancels from the allocation, so relative ratios suffice (floored to stay positive)
    rel = np.exp(np.maximum(outer - outer.max(), log(np.finfo(np.float64).tiny)))
    budget = config.rollout_budget if rollout_budget_provider is None else float(rollout_budget_provider(
        RolloutBudgetContext(draws, tuple(keys), tuple(terminal), tuple(hist_caps), dict(group_caps))))
    if not (isfinite(budget) and budget > 0):
        raise ValueError("rollout budget provider must return a positive finite value")
    alloc = allocate_variance_cost_budget(outer_ratios=rel, statistics=stats, history_capacities=hist_caps,
                                          history_groups=keys, group_capacities=group_caps, rollout_budget=budget,
                                          minimum_fresh=min_fresh)
    claims = []
    for key, a, term in zip(keys, alloc, terminal):
        if term:
            claims.append(None)
            continue
        c = store.freeze_claims([key], a.history_count)[0]
        if c.count != a.history_count:
            raise RuntimeError("frozen replay inventory changed during allocation")
        claims.append(c)
    fresh_reqs: list[ReplaySampleRequest] = []
    ranges: list = []
    for k, (key, a, term) in enumerate(zip(keys, alloc, terminal)):
        if term:
            ranges.append(None)
            continue
        lo = len(fresh_reqs)
        fresh_reqs += build_fresh_replay_requests(key=key, count=a.fresh_count, rollout_length=roll, seeds=seeds,
                                                  step_index=step_index, candidate_index=k)
        ranges.append((lo, len(fresh_reqs)))
    fresh = sample_replay_records(base_policy, fresh_reqs, reward)   # one batched call for every candidate
    out = []
    tau = config.reward_temperature
    for k, (d, a, c, term, rg) in enumerate(zip(draws, alloc, claims, terminal, ranges)):
        if term:
            v = float(reward(prompt, generated_prefix + d.token_ids))
            est = ReplayWeightEstimate(v / tau, (), (v / tau,), (), ())
        else:
            est = estimate_replay_weight(base_backend=base_backend, base_policy=base_policy, registry=registry,
                                         store=store, claim=c, fresh_count=a.fresh_count, rollout_length=roll,
                                         reward=reward, reward_temperature=tau, truncation=config.truncation,
                                         seeds=seeds, step_index=step_index, candidate_index=k,
                                         precomputed_fresh_records=fresh[rg[0]:rg[1]])
        out.append(DynamicCandidate(d, a, est, d.outer_log_ratio + est.log_weight))
    lw = np.asarray([c.log_weight for c in out], dtype=np.float64)
    p = np.exp(lw - lw.max())
    sel = int(seeds.generator("dynamic_is", step_index, "select").choice(len(out), p=p / p.sum()))
    return DynamicISStep(len(generated_prefix), tuple(out), sel)


def run_dynamic_is(base_backend: AutoregressiveBackend, registry: BehaviorRegistry, store: InMemoryReplayStore,
                   prompt: TokenSequence, config: DynamicISConfig, reward: TokenReward, reward_version: str,
                   seeds: SeedStream, *, base_sampling: SamplingConfig | None = None,
                   auxiliary_proposal: CandidateProposalSource = None,
                   statistics_provider: DesignStatisticsProvider = constant_design_statistics,
                   design_prepare: DesignPreparation | None = None,
                   rollout_budget_provider: RolloutBudgetProvider | None = None,
                   reserve_policy: BehaviorPolicy | None = None) -> DynamicISResult:
    base_sampling = base_sampling or SamplingConfig()
    _full_support(base_sampling, "base candidates")
    prompt = tuple(prompt)
    base_policy = BehaviorPolicy.for_backend(base_backend, base_sampling, label="base")
    registry.register(base_policy)
    reserve_policy = reserve_policy or base_policy
    registry.register(reserve_policy)
    gen: list[int] = []
    steps = []
    written = 0
    eos = base_sampling.eos_token_id
    while len(gen) < config.total_length:
        st = dynamic_is_step(base_backend=base_backend, registry=registry, store=store, prompt=prompt,
                             generated_prefix=tuple(gen), config=config, base_sampling=base_sampling, reward=reward,
                             reward_version=reward_version, seeds=seeds, step_index=len(steps),
                             auxiliary_proposal=auxiliary_proposal, statistics_provider=statistics_provider,
                             design_prepare=design_prepare, rollout_budget_provider=rollout_budget_provider)
        gen.extend(st.selected.token_ids)
        steps.append(st)
        if eos is not None and eos in st.selected.token_ids:
            gen = gen[:gen.index(eos) + 1]
            break
        written += write_reserve_records(base_backend=base_backend, base_sampling=base_sampling,
                                         reserve_policy=reserve_policy, store=store, prompt=prompt,
                                         generated_prefix=tuple(gen), config=config, reward=reward,
                                         reward_version=reward_version, seeds=seeds, step_index=len(steps) - 1)
    return DynamicISResult(prompt, tuple(gen), tuple(steps), written)


DYNAMIC_ARMS = ("base_candidate_fixed", "replay_aware_fixed", "replay_aware_optimal")


def run_dynamic_is_arm(backend: AutoregressiveBackend, prompt: TokenSequence, *, arm: str, candidate_count: int,
                       block_size: int, total_length: int, reward: TokenReward, seeds: SeedStream,
                       reward_temperature: float = 0.5, history: int = 4, rollout_budget: float = 16.0,
                       auxiliary_mixture: float = 0.25, auxiliary_temperature: float = 1.5,
                       history_temperature: float = 1.3, base_sampling: SamplingConfig | None = None,
                       prepare: Callable[[Callable[[], tuple]], tuple] | None = None) -> DynamicISResult:
    """One prompt under one of the dynamic-IS benchmark arms.

    ``base_candidate_fixed``: base candidates only, constant design statistics.
    ``replay_aware_fixed``: a hotter auxiliary policy of the same backend mixed into the
    candidates, and before every decision ``history`` rollouts per candidate block from a
    history policy written into the store (the decision's own draws, so the step redraws
    the same blocks), constant statistics.  ``replay_aware_optimal``: the same with the
    empirical variance-cost statistics.  ``prepare`` receives each history preparation as
    a zero-argument callable and returns its records (a caller times it this way).
    """
    if arm not in DYNAMIC_ARMS:
        raise ValueError(f"unknown dynamic-IS arm {arm!r}; choose from {DYNAMIC_ARMS}")
    sampling = base_sampling or SamplingConfig()
    aware = arm != "base_candidate_fixed"
    cfg = DynamicISConfig(candidate_count=candidate_count, block_size=block_size, total_length=total_length,
                          reward_temperature=reward_temperature, max_history_per_candidate=history if aware else 0,
                          rollout_budget=rollout_budget, auxiliary_mixture=auxiliary_mixture if aware else 0.0)
    stats = empirical_design_statistics if arm == "replay_aware_optimal" else constant_design_statistics
    hot = CandidateProposal.for_backend(backend, replace(sampling, temperature=auxiliary_temperature), label="hot")
    hist_policy = BehaviorPolicy.for_backend(backend, replace(sampling, temperature=history_temperature),
                                             label="history")
    registry, store = BehaviorRegistry([hist_policy]), InMemoryReplayStore()
    prompt = tuple(prompt)
    generated: tuple = ()
    steps: list[DynamicISStep] = []
    while len(generated) < total_length:
        k = len(steps)
        b = min(block_size, total_length - len(generated))
        rollout = total_length - len(generated) - b
        if aware and rollout > 0:
            def make(k=k, b=b, rollout=rollout, generated=generated):
                draws = draw_candidates(base_backend=backend, base_sampling=sampling, prefix=prompt + generated,
                                        count=candidate_count, block=b, mixture=cfg.auxiliary_mixture, source=hot,
                                        seeds=seeds, step=k)
                keys = dict.fromkeys(ReplayKey(prompt, generated, d.token_ids, "reward") for d in draws)
                reqs = [ReplaySampleRequest(key, rollout, seeds.derive("history", k, j, h), f"history:{k}:{j}:{h}")
                        for j, key in enumerate(keys) for h in range(history)]
                return sample_replay_records(hist_policy, reqs, reward)

            for r in (prepare(make) if prepare is not None else make()):
                store.add_evaluation(r)
        st = dynamic_is_step(base_backend=backend, registry=registry, store=store, prompt=prompt,
                             generated_prefix=generated, config=cfg, base_sampling=sampling, reward=reward,
                             reward_version="reward", seeds=seeds, step_index=k,
                             auxiliary_proposal=hot if aware else None, statistics_provider=stats)
        steps.append(st)
        generated += tuple(st.selected.token_ids)
        if sampling.eos_token_id is not None and sampling.eos_token_id in st.selected.token_ids:
            break
    return DynamicISResult(prompt, generated, tuple(steps), 0)


__all__ = ["CandidateProposal", "CandidateProposalFactory", "CandidateProposalSource", "DesignPreparation",
           "DesignStatisticsContext", "DesignStatisticsProvider", "DynamicCandidate", "DynamicCandidateDraw",
           "DynamicISResult", "DynamicISStep", "RolloutBudgetContext", "RolloutBudgetProvider",
           "DYNAMIC_ARMS", "constant_design_statistics", "draw_candidates", "dynamic_is_step",
           "empirical_design_statistics", "run_dynamic_is", "run_dynamic_is_arm"]
