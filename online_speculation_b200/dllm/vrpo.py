"""Variance-reduced masked-diffusion ELBO and the VRPO (ELBO-DPO) preference loss.

Reference behaviour: src/inference_scaling/dllm/vrpo.py:56-304.

* Mask plan: ``timestep_samples`` mask counts drawn uniformly from
  1..|answer|, each with ``masks_per_timestep`` independent uniform position
  subsets (the fixed-budget optimum is one mask per timestep).
* ELBO estimate: mean over the plan of -sum_masked CE / (mask_count / |answer|),
  with the answer's masked positions replaced by the mask token.
* VRPO shares the plan between the current and reference policies
  ("antithetic": same timesteps and same masks); the loss is
  -log sigmoid(beta [(E_cur(y_w) - E_ref(y_w)) - (E_cur(y_l) - E_ref(y_l))]).

A model may expose ``masked_logprobs(tokens [R, L], flat_index [n], targets [n],
cfg_scale=0)`` (the sm_100a LoRA policy: logits only at masked rows, fused
head + log-probability); otherwise it is called as a PyTorch module returning
full logits.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch
import torch.nn.functional as F

from ..shared.rng import SeedStream
from ..shared.types import TokenSequence
from .config import VRPOSamplingConfig


@dataclass(frozen=True, slots=True)
class VRPOMaskSample:
    timestep_index: int
    mask_count: int
    positions: tuple[int, ...]

    def __post_init__(self) -> None:
        if self.timestep_index < 0:
            raise ValueError("timestep_index must be non-negative")
        if self.mask_count <= 0 or len(self.positions) != self.mask_count:
            raise ValueError("positions must contain exactly mask_count (> 0) entries")
        if any(b <= a for a, b in zip(self.positions, self.positions[1:])):
            raise ValueError("masked positions must be sorted and unique")


@dataclass(frozen=True, slots=True)
class VRPOMaskPlan:
    answer_length: int
    timestep_samples: int
    masks_per_timestep: int
    samples: tuple[VRPOMaskSample, ...]

    def __post_init__(self) -> None:
        if self.answer_length <= 0:
            raise ValueError("answer_length must be positive")
        if len(self.samples) != self.timestep_samples * self.masks_per_timestep:
            raise ValueError("mask plan size does not match its Monte Carlo layout")
        if any(not 0 <= p < self.answer_length for s in self.samples for p in s.positions):
            raise ValueError("masked position lies outside the answer")


def sample_vrpo_mask_plan(answer_length: int, config: VRPOSamplingConfig, rng: np.random.Generator) -> VRPOMaskPlan:
    if answer_length <= 0:
        raise ValueError("answer_length must be positive")
    samples = []
    for t in range(config.timestep_samples):
        count = int(rng.integers(1, answer_length + 1))
        for _ in range(config.masks_per_timestep):
            pos = tuple(sorted(int(v) for v in rng.choice(answer_length, size=count, replace=False)))
            samples.append(VRPOMaskSample(t, count, pos))
    return VRPOMaskPlan(answer_length, config.timestep_samples, config.masks_per_timestep, tuple(samples))


def _device(model) -> torch.device:
    dev = getattr(model, "device", None)
    if dev is not None:
        return torch.device(dev)
    try:
        return next(model.parameters()).device
    except (StopIteration, AttributeError, TypeError):
        return torch.device("cpu")


def estimate_masked_elbo(model: Any, *, prompt: TokenSequence, answer: TokenSequence, mask_token_id: int,
                         plan: VRPOMaskPlan, cfg_scale: float = 0.0) -> torch.Tensor:
    """Differentiable Monte Carlo estimate of the conditional ELBO of ``answer`` given ``prompt``."""
    if len(answer) != plan.answer_length:
        raise ValueError("answer length and mask plan do not match")
    if cfg_scale < 0:
        raise ValueError("cfg_scale must be non-negative")
    dev = _device(model)
    P = len(prompt)
    full = torch.tensor(tuple(prompt) + tuple(answer), dtype=torch.long, device=dev)
    S, L = len(plan.samples), full.numel()
    batch = full.unsqueeze(0).repeat(S, 1)
    rows = torch.tensor([r for r, s in enumerate(plan.samples) for _ in s.positions], dtype=torch.long, device=dev)
    cols = torch.tensor([P + p for s in plan.samples for p in s.positions], dtype=torch.long, device=dev)
    corrupted = batch.clone()
    corrupted[rows, cols] = mask_token_id
    targets = batch[rows, cols]
    if hasattr(model, "masked_logprobs"):
        unc = None
        if cfg_scale > 0:
            unc = corrupted.clone()
            unc[:, :P] = mask_token_id
        logp = model.masked_logprobs(corrupted, rows * L + cols, targets, cfg_scale=cfg_scale, unconditional=unc)
    else:
        if cfg_scale > 0:
            unc = corrupted.clone()
            unc[:, :P] = mask_token_id
            c, u = model(torch.cat((corrupted, unc))).logits.chunk(2)
            logits = u + (cfg_scale + 1.0) * (c - u)
        else:
            logits = model(corrupted).logits
        logp = -F.cross_entropy(logits[rows, cols].float(), targets, reduction="none")
    ratio = torch.tensor([s.mask_count / plan.answer_length for s in plan.samples for _ in s.positions],
                         dtype=torch.float32, device=logp.device)
    per = torch.zeros(S, dtype=torch.float32, device=logp.device).index_add(0, rows.to(logp.device),
                                                                          logp.float() / ratio)
    return per.mean()


@dataclass(frozen=True, slots=True)
class VRPOPreferenceEstimate:
    loss: Any
    preference_score: Any
    current_chosen_elbo: Any
    reference_chosen_elbo: Any
    current_rejected_elbo: Any
    reference_rejected_elbo: Any
    current_chosen_plan: VRPOMaskPlan
    reference_chosen_plan: VRPOMaskPlan
    current_rejected_plan: VRPOMaskPlan
    reference_rejected_plan: VRPOMaskPlan


class AdapterDisabledReference:
    """The frozen base policy evaluated through an adapter model (same resident weights, adapters off).

    Works with models exposing ``disable_adapter()`` as a context manager (the
    LoRA policy here, or a PEFT model).
    """

    def __init__(self, model: Any) -> None:
        if not callable(getattr(model, "disable_adapter", None)):
            raise TypeError("model must provide a disable_adapter context")
        self.model = model
        if hasattr(model, "masked_logprobs"):
            self.masked_logprobs = self._masked_logprobs

    @property
    def device(self):
        return _device(self.model)

    def parameters(self):
        return self.model.parameters()

    def _masked_logprobs(self, *args, **kwargs):
        with self.model.disable_adapter():
            return self.model.masked_logprobs(*args, **kwargs)

    def __call__(self, *args, **kwargs):
        training = bool(getattr(self.model, "training", False))
        try:
            if hasattr(self.model, "eval"):
                self.model.eval()
            with self.model.disable_adapter():
                return self.model(*args, **kwargs)
        finally:
            if hasattr(self.model, "train"):
                self.model.train(training)


def vrpo_forward_token_slots(*, prompt_length: int, chosen_length: int, rejected_length: int,
                             config: VRPOSamplingConfig) -> dict[str, int]:
    for name, v in (("prompt_length", prompt_length), ("chosen_length", chosen_length),
                    ("rejected_length", rejected_length)):
        if v <= 0:
            raise ValueError(f"{name} must be positive")
    one = config.forward_passes * (2 * prompt_length + chosen_length + rejected_length)
    return {"current_policy": one, "reference_policy": one, "total": 2 * one}


def estimate_vrpo_preference_loss(current_model: Any, reference_model: Any, *, prompt: TokenSequence,
                                  chosen: TokenSequence, rejected: TokenSequence, mask_token_id: int,
                                  config: VRPOSamplingConfig = VRPOSamplingConfig(), beta: float = 0.2,
                                  seed: int = 0) -> VRPOPreferenceEstimate:
    if beta <= 0:
        raise ValueError("beta must be positive")
    seeds = SeedStream(seed)
    cur_w = sample_vrpo_mask_plan(len(chosen), config, seeds.generator("vrpo", "current", "chosen"))
    cur_l = sample_vrpo_mask_plan(len(rejected), config, seeds.generator("vrpo", "current", "rejected"))
    if config.antithetic:
        ref_w, ref_l = cur_w, cur_l
    else:
        ref_w = sample_vrpo_mask_plan(len(chosen), config, seeds.generator("vrpo", "reference", "chosen"))
        ref_l = sample_vrpo_mask_plan(len(rejected), config, seeds.generator("vrpo", "reference", "rejected"))
    kw = dict(prompt=prompt, mask_token_id=mask_token_id)
    cw = estimate_masked_elbo(current_model, answer=chosen, plan=cur_w, **kw)
    cl = estimate_masked_elbo(current_model, answer=rejected, plan=cur_l, **kw)
    with torch.no_grad():
        rw = estimate_masked_elbo(reference_model, answer=chosen, plan=ref_w, **kw)
        rl = estimate_masked_elbo(reference_model, answer=rejected, plan=ref_l, **kw)
    score = beta * ((cw - rw) - (cl - rl))
    return VRPOPreferenceEstimate(-F.logsigmoid(score), score, cw, rw, cl, rl, cur_w, ref_w, cur_l, ref_l)


__all__ = ["AdapterDisabledReference", "VRPOMaskPlan", "VRPOMaskSample", "VRPOPreferenceEstimate",
           "estimate_masked_elbo", "estimate_vrpo_preference_loss", "sample_vrpo_mask_plan",
           "vrpo_forward_token_slots"]
