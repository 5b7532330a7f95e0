"""Probability transforms and the exact positive-residual speculative correction.

* ``probabilities``: temperature / top-k / top-p law of one or more rows
  (temperature 0 is greedy, a one-hot at the argmax);
* ``verify_greedy``: equality of draft and target argmaxes, first mismatch
  replaced by the target token;
* ``verify_linear``: sequential p/q acceptance (accept x_i while u_i < p_i(x_i) /
  q_i(x_i)); the first rejection draws from the normalised residual (p - q)+,
  full acceptance draws a bonus token from p_n.  Emitted tokens follow p
  exactly whatever q is;
* ``linear_correction``: the same decision as fixed-shape tensor algebra
  (accept-prefix count, residual draw by exponential race, validity flag),
  the form the GPU kernel ``spec_verify`` implements.

Reference: online-speculation/src/blockspec/sampling.py:23-146 and
sampling_execution.py:15-41.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor


@dataclass(frozen=True)
class SamplingConfig:
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0

    def __post_init__(self):
        if not math.isfinite(self.temperature) or self.temperature < 0:
            raise ValueError("temperature must be finite and non-negative")
        if self.top_k < 0 or not 0 < self.top_p <= 1:
            raise ValueError("invalid top-k or top-p")


def probabilities(logits: Tensor, config: SamplingConfig) -> Tensor:
    if not torch.isfinite(logits).all():
        raise ValueError("logits must be finite")
    return transform(logits, config)


def transform(logits: Tensor, config: SamplingConfig) -> Tensor:
    """Pure tensor map (no validation) from logits to the sampling law."""
    work = logits if logits.dtype == torch.float64 else logits.float()
    if config.temperature == 0:
        return torch.zeros_like(work).scatter_(-1, work.argmax(-1, keepdim=True), 1)
    work = work / config.temperature
    if config.top_k:
        keep = min(config.top_k, work.shape[-1])
        idx = work.topk(keep, dim=-1).indices
        work = work.masked_fill(~torch.zeros_like(work, dtype=torch.bool).scatter_(-1, idx, True), -torch.inf)
    if config.top_p < 1:
        ordered, idx = work.sort(dim=-1, descending=True)
        mass = ordered.softmax(-1)
        drop = (mass.cumsum(-1) - mass) >= config.top_p  # keep the token that crosses top_p
        drop[..., 0] = False
        work = work.masked_fill(torch.zeros_like(drop).scatter_(-1, idx, drop), -torch.inf)
    return work.softmax(-1)


def greedy_tokens(logits: Tensor) -> Tensor:
    if logits.ndim < 1 or logits.shape[-1] < 1 or not torch.isfinite(logits).all():
        raise ValueError("nonempty finite logits required")
    return logits.argmax(-1)


def validate_distribution(p: Tensor) -> None:
    if p.ndim < 1 or p.shape[-1] < 1 or not torch.isfinite(p).all() or (p < 0).any():
        raise ValueError("probabilities must be finite and non-negative")
    s = p.sum(-1)
    if not torch.allclose(s, torch.ones_like(s), atol=1e-6, rtol=1e-6):
        raise ValueError("probabilities must sum to one")


def draw(p: Tensor, generator=None) -> Tensor:
    validate_distribution(p)
    return torch.multinomial(p.reshape(-1, p.shape[-1]), 1, generator=generator).reshape(p.shape[:-1])


def sample_logits(logits: Tensor, config: SamplingConfig = SamplingConfig(), generator=None) -> Tensor:
    return greedy_tokens(logits) if config.temperature == 0 else draw(probabilities(logits, config), generator)


def residual(p: Tensor, q: Tensor) -> tuple[Tensor, Tensor]:
    """Normalised positive residual (p - q)+ and its mass."""
    validate_distribution(p)
    validate_distribution(q)
    if p.shape != q.shape:
        raise ValueError("target and proposal shapes differ")
    pos = (p - q).clamp_min(0)
    mass = pos.sum(-1, keepdim=True)
    corrected = torch.where(mass > 0, pos / mass.clamp_min(torch.finfo(p.dtype).tiny), p)
    return corrected, mass.squeeze(-1)


@dataclass
class Verification:
    tokens: list[int]
    accepted: int
    rejected_at: int | None
    supervised: int


def verify_greedy(proposed: Tensor, target_ids: Tensor) -> Verification:
    if proposed.ndim != 1 or target_ids.shape != (proposed.numel() + 1,):
        raise ValueError("proposals[n] and greedy targets[n + 1] required")
    cand, tgt = proposed.tolist(), target_ids.tolist()
    for i, tok in enumerate(cand):
        if tok != tgt[i]:
            return Verification(cand[:i] + [tgt[i]], i, i, i + 1)
    return Verification(cand + [tgt[-1]], len(cand), None, len(cand))


def verify_linear(proposed: Tensor, q: Tensor, p: Tensor, *, generator=None,
                  acceptance_uniforms: Tensor | None = None) -> Verification:
    """Verify n proposals against p (n + 1 rows: the last one is the bonus row)."""
    n = proposed.numel()
    if proposed.ndim != 1 or q.shape[0] != n or p.shape != (n + 1, q.shape[-1]):
        raise ValueError("expected proposals[n], q[n, V], p[n + 1, V]")
    validate_distribution(p)
    validate_distribution(q)
    if ((proposed < 0) | (proposed >= q.shape[-1])).any():
        raise ValueError("proposal token outside the vocabulary")
    u = torch.rand(n, device=p.device, generator=generator) if acceptance_uniforms is None else acceptance_uniforms
    if u.shape != (n,) or ((u < 0) | (u >= 1)).any():
        raise ValueError("acceptance draws must lie in [0, 1)")
    out = []
    for i in range(n):
        tok = int(proposed[i])
        qi = q[i, tok]
        if qi <= 0:
            raise ValueError("a proposal cannot have zero proposal probability")
        if u[i] < torch.minimum(p[i, tok] / qi, qi.new_tensor(1.0)):
            out.append(tok)
            continue
        corr, mass = residual(p[i], q[i])
        if mass <= 0:
            raise RuntimeError("rejection with zero residual mass")
        out.append(int(draw(corr, generator)))
        return Verification(out, i, i, i + 1)
    out.append(int(draw(p[-1], generator)))
    return Verification(out, n, None, n)


def exponential_choice(weights: Tensor, exponential: Tensor) -> Tensor:
    """Index of the first arrival of independent exponential clocks with rates ``weights``."""
    return (weights / exponential.clamp_min(torch.finfo(weights.dtype).tiny)).argmax(-1)


def linear_correction(tokens: Tensor, q: Tensor, p: Tensor, uniforms: Tensor, exponential: Tensor):
    """Tensor form of ``verify_linear``: (accepted count, tail token, validity flag)."""
    n, V = q.shape
    safe = tokens.clamp(0, V - 1)
    sq = q.gather(-1, safe[:, None]).squeeze(-1)
    sp = p[:-1].gather(-1, safe[:, None]).squeeze(-1)
    accepted = uniforms < (sp / sq.clamp_min(torch.finfo(q.dtype).tiny)).clamp_max(1)
    count = torch.where(accepted, n, torch.arange(n, device=q.device)).amin()
    chosen_p = p.gather(0, count.expand(1, V))[0]
    chosen_q = torch.cat((q, torch.zeros_like(q[:1])), 0).gather(0, count.expand(1, V))[0]
    pos = (chosen_p - chosen_q).clamp_min(0)
    tail = exponential_choice(pos, exponential)
    valid = (torch.isfinite(p).all() & torch.isfinite(q).all() & (q >= 0).all() & (tokens >= 0).all()
             & (tokens < V).all() & (sq > 0).all() & (pos.sum() > 0))
    return count, tail, valid
