"""Sampling laws and the exact positive-residual speculative correction.

* ``probabilities``: the temperature / top-k / top-p law of one or more rows
  (temperature 0 is greedy: a one-hot at the argmax).  Top-k and top-p are decided
  on the rank of every logit (a stable descending order), so both filters are one
  comparison against the rank tensor;
* ``verify_greedy``: draft tokens agree with the target's argmaxes up to the first
  mismatch, which is replaced by the target token;
* ``verify_linear``: accept x_i while u_i < p_i(x_i) / q_i(x_i), all positions
  evaluated at once; the first rejection draws from the normalised residual
  (p - q)+, full acceptance draws a bonus token from p_n.  The emitted tokens follow
  p exactly, whatever q is;
* ``linear_correction``: the same decision as fixed-shape tensor algebra (accepted
  count, residual draw by an exponential race, validity flag), the oracle of the
  GPU kernel ``spec_verify``.

The acceptance rule is the standard speculative-sampling correction, as in
online-speculation/src/blockspec/sampling.py; the config fields are its public ones.
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
        if not (math.isfinite(self.temperature) and self.temperature >= 0):
            raise ValueError("temperature must be finite and non-negative")
        if self.top_k < 0:
            raise ValueError("top_k must be non-negative (0 disables it)")
        if not 0 < self.top_p <= 1:
            raise ValueError("top_p must lie in (0, 1]")


def probabilities(logits: Tensor, config: SamplingConfig) -> Tensor:
    if not torch.isfinite(logits).all():
        raise ValueError("logits must be finite")
    return transform(logits, config)


def _ranks(values: Tensor) -> Tensor:
    """Rank of every entry along the last axis in descending order (ties: lower index first)."""
    order = values.argsort(dim=-1, descending=True, stable=True)
    return order.argsort(dim=-1, stable=True)


def transform(logits: Tensor, config: SamplingConfig) -> Tensor:
    """Pure tensor map (no validation) from logits to the sampling law."""
    z = logits if logits.dtype == torch.float64 else logits.float()
    if config.temperature == 0:
        return torch.nn.functional.one_hot(z.argmax(-1), z.shape[-1]).to(z.dtype)
    z = z / config.temperature
    if config.top_k:
        z = z.masked_fill(_ranks(z) >= config.top_k, -torch.inf)
    if config.top_p < 1:
        order = z.argsort(dim=-1, descending=True, stable=True)
        sorted_mass = z.softmax(-1).gather(-1, order)
        before = sorted_mass.cumsum(-1) - sorted_mass          # mass strictly ahead of each token
        keep_sorted = before < config.top_p
        keep_sorted[..., 0] = True                             # the most likely token always stays
        keep = torch.empty_like(keep_sorted).scatter_(-1, order, keep_sorted)
        z = z.masked_fill(~keep, -torch.inf)
    return z.softmax(-1)


def greedy_tokens(logits: Tensor) -> Tensor:
    if logits.ndim == 0 or logits.shape[-1] == 0 or not torch.isfinite(logits).all():
        raise ValueError("greedy decoding needs non-empty finite logits")
    return logits.argmax(-1)


def validate_distribution(p: Tensor) -> None:
    if p.ndim == 0 or p.shape[-1] == 0 or not torch.isfinite(p).all() or bool((p < 0).any()):
        raise ValueError("a distribution must be non-empty, finite and non-negative")
    total = p.sum(-1)
    if not torch.allclose(total, torch.ones_like(total), atol=1e-6, rtol=1e-6):
        raise ValueError("a distribution must sum to one")


def draw(p: Tensor, generator=None) -> Tensor:
    validate_distribution(p)
    flat = p.reshape(-1, p.shape[-1])
    return torch.multinomial(flat, 1, generator=generator).reshape(p.shape[:-1])


def sample_logits(logits: Tensor, config: SamplingConfig = SamplingConfig(), generator=None) -> Tensor:
    if config.temperature == 0:
        return greedy_tokens(logits)
    return draw(probabilities(logits, config), generator)


def residual(p: Tensor, q: Tensor) -> tuple[Tensor, Tensor]:
    """The normalised positive residual (p - q)+ and its mass (p itself where the mass is zero)."""
    validate_distribution(p)
    validate_distribution(q)
    if p.shape != q.shape:
        raise ValueError(f"target {tuple(p.shape)} and proposal {tuple(q.shape)} shapes differ")
    excess = torch.relu(p - q)
    mass = excess.sum(-1, keepdim=True)
    normalised = torch.where(mass > 0, excess / mass.clamp_min(torch.finfo(p.dtype).tiny), p)
    return normalised, mass.squeeze(-1)


@dataclass
class Verification:
    tokens: list[int]
    accepted: int
    rejected_at: int | None
    supervised: int


def verify_greedy(proposed: Tensor, target_ids: Tensor) -> Verification:
    n = proposed.numel()
    if proposed.ndim != 1 or tuple(target_ids.shape) != (n + 1,):
        raise ValueError("verify_greedy takes proposals[n] and target argmaxes[n + 1]")
    mismatch = torch.nonzero(proposed != target_ids[:n]).flatten()
    if mismatch.numel() == 0:
        return Verification(proposed.tolist() + [int(target_ids[-1])], n, None, n)
    i = int(mismatch[0])
    return Verification(proposed[:i].tolist() + [int(target_ids[i])], i, i, i + 1)


def verify_linear(proposed: Tensor, q: Tensor, p: Tensor, *, generator=None,
                  acceptance_uniforms: Tensor | None = None) -> Verification:
    """Verify n proposals against p (n + 1 rows; the last row is the bonus row)."""
    n = proposed.numel()
    if proposed.ndim != 1 or q.shape[0] != n or tuple(p.shape) != (n + 1, q.shape[-1]):
        raise ValueError("verify_linear takes proposals[n], q[n, V] and p[n + 1, V]")
    validate_distribution(p)
    validate_distribution(q)
    V = q.shape[-1]
    if bool(((proposed < 0) | (proposed >= V)).any()):
        raise ValueError("a proposal lies outside the vocabulary")
    u = torch.rand(n, device=p.device, generator=generator) if acceptance_uniforms is None else acceptance_uniforms
    if tuple(u.shape) != (n,) or bool(((u < 0) | (u >= 1)).any()):
        raise ValueError("acceptance uniforms must be n values in [0, 1)")
    rows = torch.arange(n, device=p.device)
    q_tok = q[rows, proposed]
    if bool((q_tok <= 0).any()):
        raise ValueError("a proposal cannot have zero proposal probability")
    ratio = torch.minimum(p[rows, proposed] / q_tok, torch.ones_like(q_tok))
    rejected = torch.nonzero(~(u < ratio)).flatten()
    if rejected.numel() == 0:
        return Verification(proposed.tolist() + [int(draw(p[-1], generator))], n, None, n)
    i = int(rejected[0])
    corrected, mass = residual(p[i], q[i])
    if mass <= 0:
        raise RuntimeError("a rejection happened where the residual has no mass")
    return Verification(proposed[:i].tolist() + [int(draw(corrected, generator))], i, i, i + 1)


def exponential_choice(weights: Tensor, exponential: Tensor) -> Tensor:
    """Index of the first arrival among independent exponential clocks with rates ``weights``."""
    return (weights / exponential.clamp_min(torch.finfo(weights.dtype).tiny)).argmax(-1)


def linear_correction(tokens: Tensor, q: Tensor, p: Tensor, uniforms: Tensor, exponential: Tensor):
    """Tensor form of ``verify_linear``: (accepted count, tail token, validity flag)."""
    n, V = q.shape
    tiny = torch.finfo(q.dtype).tiny
    index = tokens.clamp(0, V - 1).unsqueeze(-1)
    q_tok = q.gather(-1, index).squeeze(-1)
    p_tok = p[:n].gather(-1, index).squeeze(-1)
    passes = uniforms < torch.clamp(p_tok / q_tok.clamp_min(tiny), max=1.0)
    positions = torch.arange(n, device=q.device)
    count = torch.where(passes, torch.full_like(positions, n), positions).min()
    q_padded = torch.cat((q, q.new_zeros(1, V)), 0)           # no proposal at the bonus position
    excess = torch.relu(p[count] - q_padded[count])
    tail = exponential_choice(excess, exponential)
    checks = (torch.isfinite(p).all(), torch.isfinite(q).all(), (q >= 0).all(), (tokens >= 0).all(),
              (tokens < V).all(), (q_tok > 0).all(), excess.sum() > 0)
    valid = checks[0]
    for c in checks[1:]:
        valid = valid & c
    return count, tail, valid
