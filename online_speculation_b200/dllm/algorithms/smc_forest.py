"""Block-diffusion SMC with a reusable forest of conditional rollouts.

Reference behaviour: src/inference_scaling/dllm/algorithms/smc_forest.py:271-359.
Particles grow one diffusion block per step.  Each particle branches
``branch_factor`` times; a branch's lookahead log-value is logmeanexp over
``rollout_count`` completions of r / tau and its incremental weight is the
telescoping difference to its parent's lookahead.  Completions a particle
already holds are reused: a stored rollout whose first block equals a branch
seeds that branch (and, with reuse, supplies branch blocks too), so only the
missing rollouts are drawn.  Systematic resampling splits the reservoirs among
the surviving copies so no rollout is counted twice.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass
from math import isfinite
from typing import Sequence

from ...shared.config import SMCForestConfig
from ...shared.importance import logmeanexp
from ...shared.rng import SeedStream
from ...shared.smc import normalize_smc_log_weights, partition_resampled_reservoirs, systematic_resample
from ...shared.types import TokenSequence
from ..config import DiffusionSamplingConfig
from ..replay import DiffusionReplayRewardBatch
from ..types import DiffusionBackend, DiffusionGenerationRequest


@dataclass(frozen=True, slots=True)
class DiffusionForestRollout:
    token_ids: TokenSequence
    reward: float


@dataclass(frozen=True, slots=True)
class DiffusionSMCParticle:
    token_ids: TokenSequence
    log_lookahead: float
    reservoir: tuple[DiffusionForestRollout, ...]
    ancestor: int


@dataclass(frozen=True, slots=True)
class DiffusionSMCBranch:
    parent_index: int
    token_ids: TokenSequence
    full_prefix: TokenSequence
    log_lookahead: float
    incremental_log_weight: float
    reservoir: tuple[DiffusionForestRollout, ...]
    reused_rollouts: int
    fresh_rollouts: int


@dataclass(frozen=True, slots=True)
class DiffusionSMCStep:
    generated_length_before: int
    branches: tuple[DiffusionSMCBranch, ...]
    normalized_weights: tuple[float, ...]
    effective_sample_size: float
    selected_branch_indices: tuple[int, ...]


@dataclass(frozen=True, slots=True)
class DiffusionSMCResult:
    prompt: TokenSequence
    token_ids: TokenSequence
    final_particles: tuple[DiffusionSMCParticle, ...]
    steps: tuple[DiffusionSMCStep, ...]
    reused_rollouts: int
    fresh_rollouts: int


def _branch_blocks(backend, prompt, particles, *, block_length: int, branch_factor: int, sampling, seeds: SeedStream,
                   step: int, reuse: bool):
    branches: list[list] = []           # [parent, block]
    inherited: list[list[DiffusionForestRollout]] = []
    reqs, where = [], []
    for pi, part in enumerate(particles):
        by_block: dict[TokenSequence, list[DiffusionForestRollout]] = defaultdict(list)
        if reuse:
            for r in part.reservoir:
                if r.token_ids[:block_length]:
                    by_block[r.token_ids[:block_length]].append(r)
        reused = [r.token_ids[:block_length] for r in part.reservoir if r.token_ids[:block_length]][:branch_factor]
        first = len(branches)
        for bi in range(branch_factor):
            branches.append([pi, reused[bi] if bi < len(reused) else ()])
            inherited.append([])
            if bi >= len(reused):
                reqs.append(DiffusionGenerationRequest(prompt + part.token_ids, block_length, sampling,
                                                       seeds.derive("dllm-smc", step, "candidate", pi, bi),
                                                       f"dllm-smc:{step}:parent:{pi}:branch:{bi}"))
                where.append(len(branches) - 1)
        slots: dict[TokenSequence, list[int]] = defaultdict(list)
        for pos in range(first, len(branches)):
            if branches[pos][1]:
                slots[branches[pos][1]].append(pos)
        for block, rolls in by_block.items():
            pos = slots.get(block)
            if pos:
                for k, r in enumerate(rolls):
                    inherited[pos[k % len(pos)]].append(DiffusionForestRollout(r.token_ids[len(block):], r.reward))
    got = backend.sample_batch(reqs) if reqs else []
    if len(got) != len(reqs):
        raise RuntimeError("backend returned an invalid SMC candidate count")
    for pos, s in zip(where, got):
        branches[pos][1] = s.token_ids
    return [tuple(b) for b in branches], inherited


def _evaluate(backend, prompt, particles, draws, inherited, *, rest: int, config: SMCForestConfig, sampling,
              reward_batch, seeds: SeedStream, step: int) -> tuple[DiffusionSMCBranch, ...]:
    tau = config.reward_temperature
    res = [list(v[:config.rollout_count]) for v in inherited]
    reqs, owner = [], []
    if rest > 0:
        for bi, ((pi, block), r) in enumerate(zip(draws, res)):
            for k in range(config.rollout_count - len(r)):
                reqs.append(DiffusionGenerationRequest(prompt + particles[pi].token_ids + block, rest, sampling,
                                                       seeds.derive("dllm-smc", step, "lookahead", bi, k),
                                                       f"dllm-smc:{step}:branch:{bi}:lookahead:{k}"))
                owner.append(bi)
    got = backend.sample_batch(reqs) if reqs else []
    if len(got) != len(reqs):
        raise RuntimeError("backend returned an invalid SMC rollout count")
    rewards = [float(v) for v in reward_batch(prompt, [particles[draws[b][0]].token_ids + draws[b][1] + s.token_ids
                                                       for b, s in zip(owner, got)])] if got else []
    if len(rewards) != len(got) or not all(isfinite(v) for v in rewards):
        raise RuntimeError("reward evaluator returned an invalid SMC rollout batch")
    for b, s, r in zip(owner, got, rewards):
        res[b].append(DiffusionForestRollout(s.token_ids, r))
    if rest == 0:
        term = [float(v) for v in reward_batch(prompt, [particles[pi].token_ids + blk for pi, blk in draws])]
        if len(term) != len(draws):
            raise RuntimeError("reward evaluator returned an invalid SMC terminal batch")
        res = [[DiffusionForestRollout((), r)] for r in term]
    out = []
    for bi, ((pi, block), r) in enumerate(zip(draws, res)):
        if not r:
            raise RuntimeError("every SMC branch requires a lookahead estimate")
        la = logmeanexp([x.reward / tau for x in r])
        reused = min(len(inherited[bi]), len(r))
        out.append(DiffusionSMCBranch(pi, block, particles[pi].token_ids + block, la,
                                      la - particles[pi].log_lookahead, tuple(r), reused,
                                      0 if rest == 0 else len(r) - reused))
    return tuple(out)


def run_diffusion_smc_rollout_forest(*, backend: DiffusionBackend, prompt: TokenSequence, config: SMCForestConfig,
                                     sampling: DiffusionSamplingConfig, reward_batch: DiffusionReplayRewardBatch,
                                     seed: int = 0) -> DiffusionSMCResult:
    sampling.validate_generation_length(config.total_length, prefix_length=len(prompt))
    sampling.validate_generation_length(config.block_size)
    seeds = SeedStream(seed)
    particles = tuple(DiffusionSMCParticle((), 0.0, (), -1) for _ in range(config.particle_count))
    steps, reused, fresh = [], 0, 0
    while len(particles[0].token_ids) < config.total_length:
        done = len(particles[0].token_ids)
        n = min(config.block_size, config.total_length - done)
        draws, inh = _branch_blocks(backend, prompt, particles, block_length=n, branch_factor=config.branch_factor,
                                    sampling=sampling, seeds=seeds, step=len(steps),
                                    reuse=config.reuse_rollout_forest)
        branches = _evaluate(backend, prompt, particles, draws, inh, rest=config.total_length - done - n,
                             config=config, sampling=sampling, reward_batch=reward_batch, seeds=seeds,
                             step=len(steps))
        probs, ess = normalize_smc_log_weights([b.incremental_log_weight for b in branches])
        sel = systematic_resample(probs, config.particle_count, seeds.generator("dllm-smc", len(steps), "resample"))
        buckets = partition_resampled_reservoirs([b.reservoir for b in branches], sel)
        particles = tuple(DiffusionSMCParticle(branches[i].full_prefix, branches[i].log_lookahead, bk, i)
                          for i, bk in zip(sel, buckets))
        reused += sum(b.reused_rollouts for b in branches)
        fresh += sum(b.fresh_rollouts for b in branches)
        steps.append(DiffusionSMCStep(done, branches, tuple(float(p) for p in probs), ess, tuple(sel)))
    k = int(seeds.generator("dllm-smc", "final").integers(len(particles)))
    return DiffusionSMCResult(prompt, particles[k].token_ids, particles, tuple(steps), reused, fresh)


__all__ = ["DiffusionForestRollout", "DiffusionSMCBranch", "DiffusionSMCParticle", "DiffusionSMCResult",
           "DiffusionSMCStep", "run_diffusion_smc_rollout_forest"]
