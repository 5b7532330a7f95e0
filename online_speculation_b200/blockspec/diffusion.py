"""Discrete corruption of draft inputs and its reverse kernels (reset-to-prior chain).

Forward process: a clean token x survives to noise level alpha (1 = clean) with
probability alpha and is otherwise replaced by a draw from a prior pi:

    q(z_alpha | x) = alpha delta_x + (1 - alpha) pi.

Between levels alpha_s > alpha_t the chain keeps the token with probability
r = alpha_t / alpha_s and otherwise resets it to the prior, so by Bayes' rule

    q(z_s = v | z_t, x) ∝ (alpha_s x_v + (1 - alpha_s) pi_v) (r [v = z_t] + (1 - r) pi_{z_t}).

:func:`posterior` evaluates that with a one-hot x (exact) or a predicted soft x
(the usual plug-in parameterisation); :func:`psi_transition` blends the ancestral
step with a corrector that first denoises fully and then re-noises to alpha_s.
:class:`UniformNoise` draws the uniform token noise that fills a draft block's
unknown positions.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/diffusion.py.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .sampling import validate_distribution


@dataclass(frozen=True)
class UniformNoise:
    """Uniform integer tokens on [low, high); ``high`` None means the vocabulary size."""

    low: int = 0
    high: int | None = None

    def __post_init__(self):
        if type(self.low) is not int or self.low < 0 or (self.high is not None and (
                type(self.high) is not int or self.high <= self.low)):
            raise ValueError("integer bounds 0 <= low < high are required")

    def sample(self, shape, vocab_size: int, *, device, generator=None) -> torch.Tensor:
        high = vocab_size if self.high is None else self.high
        if not self.low < high <= vocab_size:
            raise ValueError("the noise bounds must fit the vocabulary")
        return torch.randint(self.low, high, shape, device=device, generator=generator)


def corrupt(clean: torch.Tensor, prior: torch.Tensor, alpha: float, *, generator=None) -> torch.Tensor:
    """Keep each token with probability ``alpha``, else replace it by a draw from ``prior``."""
    validate_distribution(prior)
    if prior.ndim != 1 or not 0 <= alpha <= 1:
        raise ValueError("a one-dimensional prior and alpha in [0, 1] are required")
    fresh = torch.multinomial(prior, clean.numel(), replacement=True, generator=generator).reshape_as(clean)
    keep = torch.rand(clean.shape, device=clean.device, generator=generator) < alpha
    return torch.where(keep, clean, fresh.to(clean.dtype))


def posterior(z_t: torch.Tensor, clean: torch.Tensor, prior: torch.Tensor, alpha_s: float, alpha_t: float) -> torch.Tensor:
    """q(z_s | z_t, x) for 0 <= alpha_t < alpha_s <= 1; ``clean`` [..., V] is x (one-hot or predicted)."""
    validate_distribution(clean)
    validate_distribution(prior)
    if not 0 <= alpha_t < alpha_s <= 1:
        raise ValueError("0 <= alpha_t < alpha_s <= 1 is required")
    if prior.ndim != 1 or clean.shape[-1] != prior.numel():
        raise ValueError("the prior and the clean distribution must share the vocabulary")
    if tuple(z_t.shape) != tuple(clean.shape[:-1]):
        raise ValueError("one observed token per clean distribution is required")
    r = alpha_t / alpha_s
    keep = torch.nn.functional.one_hot(z_t.long(), prior.numel()).to(clean.dtype)
    likelihood = r * keep + (1 - r) * prior[z_t.long()][..., None]            # q(z_t | z_s = v)
    marginal = alpha_s * clean + (1 - alpha_s) * prior                          # q(z_s = v | x)
    joint = marginal * likelihood
    norm = joint.sum(-1, keepdim=True)
    if bool((norm <= 0).any()):
        raise ValueError("the noisy observation is impossible under this clean distribution")
    return joint / norm


def psi_transition(z_t: torch.Tensor, clean: torch.Tensor, prior: torch.Tensor, alpha_s: float, alpha_t: float,
                   kappa: float = 1.0) -> torch.Tensor:
    """kappa * ancestral posterior + (1 - kappa) * (denoise fully, then re-noise to alpha_s)."""
    if not 0 <= kappa <= 1:
        raise ValueError("kappa must lie in [0, 1]")
    ancestral = posterior(z_t, clean, prior, alpha_s, alpha_t)
    denoised = posterior(z_t, clean, prior, 1.0, alpha_t)
    corrector = alpha_s * denoised + (1 - alpha_s) * prior
    return kappa * ancestral + (1 - kappa) * corrector


__all__ = ["UniformNoise", "corrupt", "posterior", "psi_transition"]
