"""Offline distillation of the draft view from the frozen AR view.

Anchors are drawn at random in clean sequences.  Each anchor opens a block
``[token at the anchor, MASK x (K - 1)]`` placed at the anchor's positions; the draft
view sees the clean prefix before the anchor (the AR history of the clean sequence)
and its own block in both directions, so all blocks of a sequence train in one
forward under a block-diagonal isolation mask.  Draft row j is taught by the AR law
at the same clean position, with the full-vocabulary forward KL computed in row
chunks under activation checkpointing, so no [rows x V] tensor is kept for backward.
The layout and loss are those of online-speculation/src/blockspec/parallel/training.py
(the distillation objective of the method).
"""

from __future__ import annotations

import math
from contextlib import nullcontext
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import Tensor
from torch.utils.checkpoint import checkpoint


@dataclass
class AnchorLayout:
    tokens: Tensor        # [B, blocks * K] draft inputs (anchor token, then masks)
    positions: Tensor     # [B, blocks * K]
    allowed: Tensor       # [B, 1, blocks * K, T + blocks * K]
    teacher_rows: Tensor  # [B, blocks * (K - 1)] clean positions whose AR law teaches
    student_rows: Tensor  # [blocks * (K - 1)] draft rows that are taught


def sample_anchors(tokens: Tensor, block_size: int, count: int, *, generator=None) -> Tensor:
    if tokens.ndim != 2 or block_size < 2 or count < 1:
        raise ValueError("anchors need a [batch, time] batch, a block of at least 2 and a positive count")
    span = tokens.shape[1] - block_size + 1
    if span < 1:
        raise ValueError(f"sequences of {tokens.shape[1]} tokens cannot hold a block of {block_size}")
    return torch.randint(span, (tokens.shape[0], count), device=tokens.device, generator=generator)


def anchor_layout(tokens: Tensor, anchors: Tensor, block_size: int, mask_token_id: int) -> AnchorLayout:
    B, T = tokens.shape
    if anchors.ndim != 2 or anchors.shape[0] != B or anchors.dtype != torch.long:
        raise ValueError("anchors must be an integer [batch, blocks] tensor")
    if bool(((anchors < 0) | (anchors + block_size > T)).any()):
        raise ValueError("every anchor needs its whole block inside the sequence")
    device = tokens.device
    blocks = anchors.shape[1]
    K = block_size
    offsets = torch.arange(K, device=device)
    positions = (anchors.unsqueeze(-1) + offsets).reshape(B, blocks * K)
    inputs = torch.full((B, blocks, K), mask_token_id, dtype=tokens.dtype, device=device)
    inputs[..., 0] = torch.take_along_dim(tokens, anchors, dim=1)
    # a draft row sees the clean tokens strictly before its block's anchor ...
    anchor_of_row = anchors.repeat_interleave(K, dim=1)                               # [B, blocks * K]
    history = torch.arange(T, device=device).view(1, 1, T) < anchor_of_row.unsqueeze(-1)
    # ... and every row of its own block, nothing of the other blocks
    own_block = torch.block_diag(*[torch.ones(K, K, dtype=torch.bool, device=device)] * blocks)
    allowed = torch.cat((history, own_block.expand(B, -1, -1)), dim=-1).unsqueeze(1)
    taught = (torch.arange(blocks * K, device=device) % K) < K - 1                     # every row but the last
    student_rows = torch.nonzero(taught).flatten()
    teacher_rows = positions[:, taught]
    return AnchorLayout(inputs.reshape(B, blocks * K), positions, allowed, teacher_rows, student_rows)


def forward_kl(student_logits: Tensor, teacher_logits: Tensor) -> Tensor:
    """Mean over rows of KL(teacher || student)."""
    log_p = teacher_logits.detach().float().log_softmax(-1)
    log_q = student_logits.float().log_softmax(-1)
    return F.kl_div(log_q, log_p, reduction="none", log_target=True).sum(-1).mean()


def _chunked_kl(head: Tensor, student_hidden: Tensor, teacher_hidden: Tensor, chunk_rows: int) -> Tensor:
    """Row-weighted mean of the forward KL, one checkpointed head GEMM per chunk."""
    rows = student_hidden.shape[0]

    def piece(s: Tensor, t: Tensor) -> Tensor:
        with torch.no_grad():
            teacher = F.linear(t, head)
        return forward_kl(F.linear(s, head), teacher)

    total = student_hidden.new_zeros(())
    for start in range(0, rows, chunk_rows):
        stop = min(rows, start + chunk_rows)
        part = checkpoint(piece, student_hidden[start:stop], teacher_hidden[start:stop], use_reentrant=False)
        total = total + part * ((stop - start) / rows)
    return total


def distillation_loss(model, tokens: Tensor, anchors: Tensor, *, block_size=None, chunk_rows: int = 32,
                      draft_weights=None) -> Tensor:
    K = model.config.block_size if block_size is None else block_size
    if chunk_rows < 1:
        raise ValueError("chunk_rows has to be positive")
    trainable_shared = [n for n, p in model.named_parameters() if p.requires_grad and ".attention.draft." not in n]
    if trainable_shared:
        raise ValueError("only draft attention may train here: call train_draft_only() first "
                         f"({len(trainable_shared)} other parameters require gradients)")
    layout = anchor_layout(tokens, anchors, K, model.config.mask_token_id)
    H = model.config.hidden_size
    with torch.no_grad():
        teacher = model(tokens, compute_logits=False)
        teacher_hidden = torch.take_along_dim(teacher.hidden, layout.teacher_rows.unsqueeze(-1), dim=1)
    options = dict(view="draft", cache=teacher.cache, positions=layout.positions, allowed=layout.allowed,
                   compute_logits=False)
    if draft_weights is None:
        student = model(layout.tokens, **options)
    else:
        student = torch.func.functional_call(model, draft_weights, (layout.tokens,), options)
    student_hidden = student.hidden[:, layout.student_rows]
    return _chunked_kl(model.head.weight, student_hidden.reshape(-1, H), teacher_hidden.reshape(-1, H), chunk_rows)


def distillation_update(model, batches, optimizer, *, learning_rate: float, clip_grad: float = 1.0,
                        chunk_rows: int = 32, autocast=nullcontext, master=None) -> dict:
    """One AdamW step over fixed (tokens, anchors) micro-batches on the draft parameters."""
    if not batches:
        raise ValueError("an update needs at least one micro-batch")
    if not all(math.isfinite(v) and v > 0 for v in (learning_rate, clip_grad)):
        raise ValueError("learning_rate and clip_grad have to be finite and positive")
    resident = dict(model.named_parameters())
    draft = {n: p for n, p in resident.items() if ".attention.draft." in n}
    trained = draft if master is None else master
    owned = [p for group in optimizer.param_groups for p in group["params"]]
    if trained.keys() != draft.keys() or {id(p) for p in owned} != {id(p) for p in trained.values()}:
        raise ValueError("the optimizer must hold exactly the draft attention parameters")
    for group in optimizer.param_groups:
        group["lr"] = learning_rate
    optimizer.zero_grad(set_to_none=True)
    losses = []
    try:
        with torch.enable_grad():
            for tokens, anchors in batches:
                weights = None if master is None else {n: p.to(resident[n].dtype) for n, p in master.items()}
                with autocast():
                    loss = distillation_loss(model, tokens, anchors, chunk_rows=chunk_rows, draft_weights=weights)
                if not torch.isfinite(loss):
                    raise FloatingPointError("the distillation loss is not finite")
                (loss / len(batches)).backward()
                losses.append(float(loss.detach()))
        norm = torch.nn.utils.clip_grad_norm_(owned, clip_grad, error_if_nonfinite=True)
        optimizer.step()
    finally:
        optimizer.zero_grad(set_to_none=True)
    return {"loss": sum(losses) / len(losses), "learning_rate": learning_rate, "gradient_norm": float(norm)}
