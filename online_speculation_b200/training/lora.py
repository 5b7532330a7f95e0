"""LoRA adapters on frozen bf16 weights, with the tcgen05 GEMM for every product.

y = x W^T + s (x A^T) B^T with A [r, in], B [out, r], s = alpha / r.  The
adapter term is added through the GEMM's residual epilogue (one extra small
GEMM, no separate add).  ``groups`` splits the output rows into equal blocks
with their own (A_g, B_g), which is how a fused QKV projection carries
separate q / k / v adapters: A stacks the blocks' A_g and B is block-diagonal.

Reference: PEFT LoRA as configured in configs/gsm8k_llada_moe_3090.toml
(``[vrpo_lora]``: r 16, alpha 32, dropout 0.05) and
experiments/arllm/train_gsm8k_grpo.py:366-415.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from ..ops import kernels as K


@dataclass(frozen=True)
class LoRAConfig:
    rank: int = 16
    alpha: float = 32.0
    dropout: float = 0.0
    targets: tuple[str, ...] = ("q_proj", "k_proj", "v_proj", "o_proj")

    def __post_init__(self):
        if self.rank < 1 or self.alpha <= 0 or not 0 <= self.dropout < 1:
            raise ValueError("positive rank / alpha and dropout in [0, 1) required")

    @property
    def scale(self) -> float:
        return self.alpha / self.rank


class LoRAParameters:
    """Trainable A / B of one (possibly grouped) projection, as fp32 tensors requiring grad."""

    def __init__(self, in_features: int, out_features: int, rank: int, groups: int = 1, *, device="cpu",
                 generator: torch.Generator | None = None):
        if out_features % groups:
            raise ValueError("output rows must split evenly into groups")
        self.in_features, self.out_features, self.rank, self.groups = in_features, out_features, rank, groups
        bound = 1.0 / math.sqrt(in_features)       # kaiming-uniform(a = sqrt(5)) bound, as PEFT initialises A
        a = (torch.rand(groups * rank, in_features, generator=generator) * 2 - 1) * bound
        self.A = a.to(device).requires_grad_(True)
        self.B = torch.zeros(out_features, groups * rank, device=device, requires_grad=True)  # B = 0: no-op at start
        per = out_features // groups
        mask = torch.zeros(out_features, groups * rank, device=device)
        for g in range(groups):
            mask[g * per:(g + 1) * per, g * rank:(g + 1) * rank] = 1
        self.block_mask = mask

    def parameters(self) -> list[torch.Tensor]:
        return [self.A, self.B]


class _LoRALinear(torch.autograd.Function):
    """y = x W^T (+ bias) + s (xa A^T) (B * mask)^T.  ``xa`` is the adapter's input
    (x itself, or x after dropout); gradients flow to both."""

    @staticmethod
    def forward(ctx, x, xa, A, B, w, bias, scale, mask):
        xb = x.to(torch.bfloat16).contiguous()
        xab = xb if xa is x else xa.to(torch.bfloat16).contiguous()
        Ab = A.to(torch.bfloat16).contiguous()
        Bb = (B * mask).to(torch.bfloat16).contiguous()
        u = K.linear(xab, Ab)                                         # [T, g r]
        y = K.linear(xb, w, bias=bias)
        us = (u.float() * scale).to(torch.bfloat16)
        K.linear(us, Bb, residual=y, out=y)                           # y += s u B^T
        ctx.save_for_backward(xab, Ab, Bb, u, w, mask)
        ctx.scale = scale
        ctx.same = xa is x
        return y

    @staticmethod
    def backward(ctx, gy):
        xab, Ab, Bb, u, w, mask = ctx.saved_tensors
        s = ctx.scale
        gy = gy.to(torch.bfloat16).contiguous()
        gu = K.linear(gy, Bb.t().contiguous(), out_dtype=torch.float32) * s        # [T, g r]
        gB = K.linear(K.transpose_padded(gy), K.transpose_padded((u.float() * s).to(torch.bfloat16)),
                      out_dtype=torch.float32) * mask                               # [out, g r]
        gub = gu.to(torch.bfloat16).contiguous()
        gA = K.linear(K.transpose_padded(gub), K.transpose_padded(xab), out_dtype=torch.float32)  # [g r, in]
        gx = K.linear(gy, w.t().contiguous())
        if ctx.same:
            K.linear(gub, Ab.t().contiguous(), residual=gx, out=gx)                 # gx += gu A
            return gx, None, gA, gB, None, None, None, None
        gxa = K.linear(gub, Ab.t().contiguous())
        return gx, gxa, gA, gB, None, None, None, None


def lora_linear(x: torch.Tensor, w: torch.Tensor, lora: LoRAParameters | None, scale: float,
                bias: torch.Tensor | None = None, *, dropout: float = 0.0, training: bool = False) -> torch.Tensor:
    """Frozen ``w`` (+ bias) plus the adapter; plain kernel linear when ``lora`` is None.

    Dropout (training only) acts on the adapter's input, as in PEFT; the frozen
    product always sees the undropped input and passes its gradient on.
    """
    if lora is None:
        return K.linear(x, w, bias=bias) if x.is_cuda else K.linear_reference(x, w, bias=bias).to(torch.bfloat16)
    xa = torch.nn.functional.dropout(x.float(), dropout, True).to(x.dtype) if dropout > 0 and training else x
    if x.is_cuda:
        return _LoRALinear.apply(x, xa, lora.A, lora.B, w, bias, float(scale), lora.block_mask)
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    return (y + scale * (xa.float() @ lora.A.t()) @ (lora.B * lora.block_mask).t()).to(torch.bfloat16)
