"""Trajectory-power MH and sampled block beam search for exact diffusion policies.

Reference behaviour: src/inference_scaling/dllm/algorithms/search.py:87-431.

* Power MH targets p(trace | prompt)^alpha.  The final-token marginal is
  intractable but a reverse trajectory's density is exact, so cuts fall on
  diffusion-block boundaries: the suffix after a uniformly drawn block is
  redrawn from a tempered proposal (temperature / alpha by default) and the
  Hastings ratio uses the base and proposal densities of the old and new
  suffix blocks.  Stages grow the continuation one decision block at a time.
* Block beam keeps the ``width`` highest trajectory densities at every
  decision-block boundary (``width`` draws from the root, then
  ``branching_factor`` per retained beam).
"""

from __future__ import annotations

from dataclasses import dataclass, replace

from ...shared.mh import decide_metropolis_hastings
from ...shared.rng import SeedStream
from ...shared.types import TokenSequence
from ..config import DiffusionBlockBeamConfig, DiffusionPowerMHConfig, DiffusionSamplingConfig, \
    diffusion_decision_stage_lengths
from ..types import DiffusionBackend, DiffusionGenerationRequest, DiffusionSample, DiffusionTraceStep, \
    DiffusionTrajectoryScoreRequest


def exact_logprob(sample: DiffusionSample) -> float:
    if sample.trajectory_logprob is None:
        raise ValueError("an exact diffusion trajectory density is required")
    return float(sample.trajectory_logprob)


@dataclass(frozen=True, slots=True)
class DiffusionPowerMHBlock:
    sample: DiffusionSample
    base_trajectory_logprob: float
    proposal_trajectory_logprob: float


@dataclass(frozen=True, slots=True)
class DiffusionPowerMHState:
    prompt: TokenSequence
    blocks: tuple[DiffusionPowerMHBlock, ...]

    @property
    def token_ids(self) -> TokenSequence:
        return tuple(t for b in self.blocks for t in b.sample.token_ids)

    @property
    def base_trajectory_logprob(self) -> float:
        return sum(b.base_trajectory_logprob for b in self.blocks)

    @property
    def proposal_trajectory_logprob(self) -> float:
        return sum(b.proposal_trajectory_logprob for b in self.blocks)


@dataclass(frozen=True, slots=True)
class DiffusionPowerMHStep:
    stage_length: int
    update: int
    cut: int
    proposal: DiffusionSample
    previous_base_trajectory_logprob: float
    proposed_base_trajectory_logprob: float
    previous_proposal_trajectory_logprob: float
    proposed_proposal_trajectory_logprob: float
    log_acceptance: float
    acceptance_probability: float
    accepted: bool


@dataclass(frozen=True, slots=True)
class DiffusionPowerMHResult:
    prompt: TokenSequence
    alpha: float
    initial: DiffusionPowerMHState
    steps: tuple[DiffusionPowerMHStep, ...]
    final: DiffusionPowerMHState

    @property
    def acceptance_rate(self) -> float:
        return sum(s.accepted for s in self.steps) / len(self.steps) if self.steps else 0.0


def split_into_blocks(sample: DiffusionSample, sampling: DiffusionSamplingConfig) -> tuple[DiffusionSample, ...]:
    """One exact suffix sample -> independently scoreable per-block samples."""
    exact_logprob(sample)
    blocks, off = [], 0
    while off < len(sample.token_ids):
        n = min(sampling.block_length, len(sample.token_ids) - off)
        b = len(blocks)
        trace = tuple(DiffusionTraceStep(0, s.step_index, tuple(p - off for p in s.positions), s.token_ids, s.logprob)
                      for s in sample.trace if s.block_index == b)
        if not trace:
            raise RuntimeError("an exact trajectory omitted a generated diffusion block")
        blocks.append(DiffusionSample(sample.prefix + sample.token_ids[:off], sample.token_ids[off:off + n], trace,
                                      sum(float(s.logprob) for s in trace), sample.policy_id, sample.model_id,
                                      f"{sample.request_id}:block:{b}", sample.finish_reason))
        off += n
    return tuple(blocks)


def _sample_suffix(backend, prefix, length, base: DiffusionSamplingConfig, prop: DiffusionSamplingConfig, seed: int,
                   request_id: str):
    got = backend.sample_batch([DiffusionGenerationRequest(prefix, length, prop, seed, request_id)])
    if len(got) != 1:
        raise RuntimeError("backend returned an invalid number of power-MH suffixes")
    blocks = split_into_blocks(got[0], prop)
    if base.policy_id == prop.policy_id:
        scores = [float(b.trajectory_logprob) for b in blocks]
    else:
        scores = backend.score_trajectories([DiffusionTrajectoryScoreRequest(b, base) for b in blocks])
    if len(scores) != len(blocks):
        raise RuntimeError("backend returned an invalid number of power-MH block scores")
    return got[0], tuple(DiffusionPowerMHBlock(b, float(s), exact_logprob(b)) for b, s in zip(blocks, scores))


def _full_support_exact(s: DiffusionSamplingConfig, what: str) -> None:
    if not s.has_exact_trajectory_density:
        raise ValueError(f"trajectory-power MH requires an exact {what} policy")
    if s.top_k or s.top_p < 1:
        raise ValueError(f"trajectory-power MH requires a full-support {what}")


def run_diffusion_trajectory_power_mh(*, backend: DiffusionBackend, prompt: TokenSequence,
                                      config: DiffusionPowerMHConfig, sampling: DiffusionSamplingConfig,
                                      proposal_sampling: DiffusionSamplingConfig | None = None,
                                      seed: int = 0) -> DiffusionPowerMHResult:
    _full_support_exact(sampling, "base")
    prop = proposal_sampling or replace(sampling, temperature=sampling.temperature / config.alpha)
    _full_support_exact(prop, "proposal")
    key = lambda s: (s.block_length, s.steps_per_block, s.remasking, s.mask_token_id)  # noqa: E731
    if key(sampling) != key(prop):
        raise ValueError("base and proposal trajectory schedules must match")
    stages = diffusion_decision_stage_lengths(prompt_length=len(prompt), total_length=config.total_length,
                                              decision_block_size=config.decision_block_size, sampling=sampling)
    seeds = SeedStream(seed)
    cur = DiffusionPowerMHState(prompt, ())
    initial, steps, length, g = None, [], 0, 0
    for si, ext in enumerate(stages):
        _, blocks = _sample_suffix(backend, prompt + cur.token_ids, ext, sampling, prop,
                                   seeds.derive("dllm-power-mh", si, "extend"), f"dllm-power-mh:stage:{si}:extend")
        cur = DiffusionPowerMHState(prompt, cur.blocks + blocks)
        length += ext
        initial = initial or cur
        for u in range(config.updates_per_stage):
            g += 1
            cut_block = int(seeds.generator("dllm-power-mh", si, u, "cut").integers(0, len(cur.blocks)))
            kept, old = cur.blocks[:cut_block], cur.blocks[cut_block:]
            cut = sum(len(b.sample.token_ids) for b in kept)
            proposal, new = _sample_suffix(backend, prompt + cur.token_ids[:cut], length - cut, sampling, prop,
                                           seeds.derive("dllm-power-mh", si, u, "proposal"),
                                           f"dllm-power-mh:stage:{si}:update:{u}")
            old_p = sum(b.base_trajectory_logprob for b in old)
            old_q = sum(b.proposal_trajectory_logprob for b in old)
            new_p = sum(b.base_trajectory_logprob for b in new)
            new_q = sum(b.proposal_trajectory_logprob for b in new)
            d = decide_metropolis_hastings(current_target_log_density=config.alpha * old_p,
                                           proposed_target_log_density=config.alpha * new_p,
                                           forward_proposal_log_probability=new_q,
                                           reverse_proposal_log_probability=old_q,
                                           uniform=float(seeds.generator("dllm-power-mh", si, u, "accept").random()))
            if d.accepted:
                cur = DiffusionPowerMHState(prompt, kept + new)
            steps.append(DiffusionPowerMHStep(length, g, cut, proposal, old_p, new_p, old_q, new_q, d.log_acceptance,
                                              d.acceptance_probability, d.accepted))
    return DiffusionPowerMHResult(prompt, config.alpha, initial, tuple(steps), cur)


@dataclass(frozen=True, slots=True)
class DiffusionBeamHypothesis:
    token_ids: TokenSequence
    trajectory_logprob: float
    samples: tuple[DiffusionSample, ...]


@dataclass(frozen=True, slots=True)
class DiffusionBlockBeamStage:
    generated_length_before: int
    proposals: int
    retained: tuple[DiffusionBeamHypothesis, ...]


@dataclass(frozen=True, slots=True)
class DiffusionBlockBeamResult:
    prompt: TokenSequence
    stages: tuple[DiffusionBlockBeamStage, ...]
    beams: tuple[DiffusionBeamHypothesis, ...]

    @property
    def best(self) -> DiffusionBeamHypothesis:
        return self.beams[0]


def run_diffusion_block_beam(*, backend: DiffusionBackend, prompt: TokenSequence, config: DiffusionBlockBeamConfig,
                             sampling: DiffusionSamplingConfig, seed: int = 0) -> DiffusionBlockBeamResult:
    if not sampling.has_exact_trajectory_density:
        raise ValueError("block beam search requires an exact diffusion policy")
    seeds = SeedStream(seed)
    beams = (DiffusionBeamHypothesis((), 0.0, ()),)
    stages, done = [], 0
    lengths = diffusion_decision_stage_lengths(prompt_length=len(prompt), total_length=config.total_length,
                                               decision_block_size=config.decision_block_size, sampling=sampling)
    for si, n in enumerate(lengths):
        per = config.width if si == 0 else config.branching_factor
        reqs, owners = [], []
        for bi, beam in enumerate(beams):
            for d in range(per):
                reqs.append(DiffusionGenerationRequest(prompt + beam.token_ids, n, sampling,
                                                       seeds.derive("dllm-block-beam", si, bi, d),
                                                       f"dllm-block-beam:stage:{si}:beam:{bi}:draw:{d}"))
                owners.append(bi)
        got = backend.sample_batch(reqs)
        if len(got) != len(reqs):
            raise RuntimeError("backend returned an invalid number of beam proposals")
        grown = [DiffusionBeamHypothesis(beams[o].token_ids + s.token_ids,
                                         beams[o].trajectory_logprob + exact_logprob(s), beams[o].samples + (s,))
                 for o, s in zip(owners, got)]
        grown.sort(key=lambda h: (h.trajectory_logprob, h.token_ids), reverse=True)
        beams = tuple(grown[:config.width])
        stages.append(DiffusionBlockBeamStage(done, len(grown), beams))
        done += n
    return DiffusionBlockBeamResult(prompt, tuple(stages), beams)


__all__ = ["DiffusionBeamHypothesis", "DiffusionBlockBeamResult", "DiffusionBlockBeamStage", "DiffusionPowerMHBlock",
           "DiffusionPowerMHResult", "DiffusionPowerMHState", "DiffusionPowerMHStep", "exact_logprob",
           "run_diffusion_block_beam", "run_diffusion_trajectory_power_mh", "split_into_blocks"]
