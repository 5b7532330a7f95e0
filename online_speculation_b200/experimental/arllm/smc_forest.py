"""Sequential Monte Carlo over blocks with a reusable rollout forest.

Particles grow one base-model block at a time.  A positive rollout estimate
h(prefix) = mean exp(r / tau) over base-conditional completions twists the
weights; a branch's incremental weight is h(child) / h(parent), so the factors
telescope to the final target p(y) exp(r(y) / tau).  A completion sampled for
the parent's estimate whose first block equals a child's block is itself a
valid base-conditional completion of that child, so it is carried forward
(the matching suffix) instead of being re-sampled; reservoirs of duplicated
particles are split, never copied, and missing entries are topped up with
fresh rollouts.  Rewards can stream: each completion's reward starts on a
worker as soon as the backend finishes it.

Reference behaviour: src/inference_scaling/experimental/arllm/smc_forest.py:44-434.
"""

from __future__ import annotations

from collections import defaultdict
from collections.abc import Sequence
from dataclasses import dataclass
from math import isfinite

from ...arllm.acceleration import StreamingRewardEvaluator
from ...arllm.algorithms.conditional_is import TokenBatchReward, TokenReward, _full_support
from ...arllm.config import SamplingConfig, SMCForestConfig
from ...arllm.types import AutoregressiveBackend, GenerationRequest
from ...shared.importance import logmeanexp
from ...shared.rng import SeedStream
from ...shared.smc import normalize_smc_log_weights, partition_resampled_reservoirs, systematic_resample
from ...shared.types import TokenSequence


@dataclass(frozen=True, slots=True)
class ForestRollout:
    token_ids: TokenSequence      # base-conditional completion after the owner's prefix
    reward: float                 # reward of the full sequence it completes


@dataclass(frozen=True, slots=True)
class SMCParticle:
    token_ids: TokenSequence
    log_lookahead: float
    reservoir: tuple[ForestRollout, ...]
    ancestor: int


@dataclass(frozen=True, slots=True)
class SMCBranch:
    parent_index: int
    token_ids: TokenSequence
    full_prefix: TokenSequence
    log_lookahead: float
    incremental_log_weight: float
    reservoir: tuple[ForestRollout, ...]
    reused_rollouts: int
    fresh_rollouts: int


@dataclass(frozen=True, slots=True)
class SMCForestStep:
    generated_length_before: int
    branches: tuple[SMCBranch, ...]
    normalized_weights: tuple[float, ...]
    effective_sample_size: float
    selected_branch_indices: tuple[int, ...]


@dataclass(frozen=True, slots=True)
class SMCForestResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    final_particles: tuple[SMCParticle, ...]
    steps: tuple[SMCForestStep, ...]
    reused_rollouts: int
    fresh_rollouts: int


def _propose_blocks(backend, prompt, particles, *, block, branch_factor, sampling, seeds, step, reuse):
    """Child blocks per particle: first the blocks its reservoir already starts with, then fresh draws.

    Returns (parent, block) per branch and the completions each branch inherits.
    """
    eos = sampling.eos_token_id
    branches: list[list] = []
    inherited: list[list[ForestRollout]] = []
    reqs, slots = [], []
    for pi, part in enumerate(particles):
        if eos is not None and eos in part.token_ids:
            for _ in range(branch_factor):
                branches.append([pi, ()])
                inherited.append(list(part.reservoir))
            continue
        first = len(branches)
        starts = [r.token_ids[:block] for r in part.reservoir if r.token_ids[:block]]
        for bi in range(branch_factor):
            inherited.append([])
            if bi < len(starts):
                branches.append([pi, starts[bi]])
                continue
            branches.append([pi, ()])
            reqs.append(GenerationRequest(prompt + part.token_ids, block, sampling,
                                          seeds.derive("smc_forest", step, "candidate", pi, bi),
                                          f"smc-forest:step:{step}:parent:{pi}:branch:{bi}"))
            slots.append(first + bi)
        if reuse:
            # deal each matching completion to the children with that block, round-robin
            owners: dict[TokenSequence, list[int]] = defaultdict(list)
            for pos in range(first, first + branch_factor):
                if branches[pos][1]:
                    owners[branches[pos][1]].append(pos)
            dealt: dict[TokenSequence, int] = defaultdict(int)
            for r in part.reservoir:
                blk = r.token_ids[:block]
                if blk and owners.get(blk):
                    tgt = owners[blk][dealt[blk] % len(owners[blk])]
                    dealt[blk] += 1
                    inherited[tgt].append(ForestRollout(r.token_ids[len(blk):], r.reward))
    if reqs:
        got = backend.sample_batch(reqs)
        if len(got) != len(reqs):
            raise RuntimeError("base backend returned an invalid candidate count")
        for pos, smp in zip(slots, got):
            if not smp.token_ids:
                raise RuntimeError("SMC candidate blocks must be nonempty")
            branches[pos][1] = tuple(smp.token_ids)
    return [tuple(b) for b in branches], inherited


def _reward_values(prompt, seqs, reward, reward_batch):
    if reward_batch is not None:
        vals = [float(v) for v in reward_batch(prompt, list(seqs))]
        if len(vals) != len(seqs):
            raise ValueError("reward_batch returned an invalid number of rewards")
    else:
        if reward is None:
            raise ValueError("a reward callback is required")
        vals = [float(reward(prompt, s)) for s in seqs]
    if any(not isfinite(v) for v in vals):
        raise ValueError("reward must be finite")
    return vals


def _evaluate(backend, prompt, particles, draws, inherited, *, rest, config, sampling, reward, reward_batch, seeds,
              step, evaluator) -> tuple[SMCBranch, ...]:
    eos = sampling.eos_token_id
    res = [list(v[:config.rollout_count]) for v in inherited]
    reqs, owner, inputs, terminal = [], [], [], []
    for bi, (pi, blk) in enumerate(draws):
        pre = particles[pi].token_ids + blk
        if rest == 0 or (eos is not None and (eos in particles[pi].token_ids or eos in blk)):
            terminal.append(bi)
            continue
        for ri in range(config.rollout_count - len(res[bi])):
            reqs.append(GenerationRequest(prompt + pre, rest, sampling,
                                          seeds.derive("smc_forest", step, "lookahead", bi, ri),
                                          f"smc-forest:step:{step}:branch:{bi}:rollout:{ri}"))
            owner.append(bi)
            inputs.append((prompt, pre))
    if reqs and evaluator is not None:
        if reward is None or reward_batch is not None:
            raise ValueError("streaming SMC rewards require a scalar reward callback")
        samples, rewards, _ = evaluator.sample_and_score(backend, reqs, inputs, reward)
        rewards = [float(v) for v in rewards]
        if any(not isfinite(v) for v in rewards):
            raise ValueError("reward must be finite")
    else:
        samples = backend.sample_batch(reqs) if reqs else []
        rewards = _reward_values(prompt, [p + s.token_ids for (_, p), s in zip(inputs, samples)], reward,
                                 reward_batch) if reqs else []
    if len(samples) != len(reqs) or len(rewards) != len(reqs):
        raise RuntimeError("SMC rollout or reward count is invalid")
    for bi, smp, v in zip(owner, samples, rewards):
        res[bi].append(ForestRollout(tuple(smp.token_ids), v))
    for bi in terminal:
        pi, blk = draws[bi]
        res[bi] = [ForestRollout((), _reward_values(prompt, [particles[pi].token_ids + blk], reward,
                                                    reward_batch)[0])]
    out = []
    term = set(terminal)
    for bi, (pi, blk) in enumerate(draws):
        if not res[bi]:
            raise RuntimeError("each SMC branch needs a positive lookahead estimate")
        lh = logmeanexp([r.reward / config.reward_temperature for r in res[bi]])
        reused = min(len(inherited[bi]), len(res[bi]))
        out.append(SMCBranch(pi, blk, particles[pi].token_ids + blk, lh, lh - particles[pi].log_lookahead,
                             tuple(res[bi]), reused, 0 if bi in term else len(res[bi]) - reused))
    return tuple(out)


def run_smc_rollout_forest(base_backend: AutoregressiveBackend, prompt: TokenSequence, config: SMCForestConfig,
                           reward: TokenReward | None, seeds: SeedStream, *,
                           base_sampling: SamplingConfig | None = None,
                           reward_batch: TokenBatchReward | None = None,
                           streaming_rewards: bool = True) -> SMCForestResult:
    sampling = base_sampling or SamplingConfig()
    _full_support(sampling, "base candidates")
    if (reward is None) == (reward_batch is None):
        raise ValueError("provide exactly one of reward or reward_batch")
    prompt = tuple(prompt)
    eos = sampling.eos_token_id
    particles = tuple(SMCParticle((), 0.0, (), -1) for _ in range(config.particle_count))
    evaluator = (StreamingRewardEvaluator(workers=config.reward_workers)
                 if streaming_rewards and reward is not None and reward_batch is None else None)
    steps, reused, fresh = [], 0, 0
    try:
        while max(len(p.token_ids) for p in particles) < config.total_length and not (
                eos is not None and all(eos in p.token_ids for p in particles)):
            before = max(len(p.token_ids) for p in particles)
            block = min(config.block_size, config.total_length - before)
            draws, inh = _propose_blocks(base_backend, prompt, particles, block=block,
                                         branch_factor=config.branch_factor, sampling=sampling, seeds=seeds,
                                         step=len(steps), reuse=config.reuse_rollout_forest)
            branches = _evaluate(base_backend, prompt, particles, draws, inh,
                                 rest=max(0, config.total_length - before - block), config=config,
                                 sampling=sampling, reward=reward, reward_batch=reward_batch, seeds=seeds,
                                 step=len(steps), evaluator=evaluator)
            probs, ess = normalize_smc_log_weights([b.incremental_log_weight for b in branches])
            sel = systematic_resample(probs, config.particle_count,
                                      seeds.generator("smc_forest", len(steps), "resample"))
            buckets = partition_resampled_reservoirs([b.reservoir for b in branches], sel)
            particles = tuple(SMCParticle(branches[i].full_prefix, branches[i].log_lookahead, bk, i)
                              for i, bk in zip(sel, buckets))
            reused += sum(b.reused_rollouts for b in branches)
            fresh += sum(b.fresh_rollouts for b in branches)
            steps.append(SMCForestStep(before, branches, probs, ess, sel))
    finally:
        if evaluator is not None:
            evaluator.close()
    out = particles[int(seeds.generator("smc_forest", "final").integers(len(particles)))].token_ids
    if eos is not None and eos in out:
        out = out[:out.index(eos) + 1]
    return SMCForestResult(prompt, out, particles, tuple(steps), reused, fresh)


__all__ = ["ForestRollout", "SMCBranch", "SMCForestResult", "SMCForestStep", "SMCParticle", "run_smc_rollout_forest"]
