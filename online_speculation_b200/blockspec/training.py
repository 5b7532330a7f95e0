"""Offline block distillation of the draft view from the frozen AR view.

Random anchors are drawn in clean sequences; each anchor opens a block
``[token_at_anchor, MASK x (K-1)]`` placed at the anchor's positions.  The
draft view sees the clean prefix before its anchor (AR history of the clean
sequence) plus its own block bidirectionally, so many blocks of one sequence
train in one forward with an isolation mask.  The teacher for draft row j is
the AR distribution at the same clean position.  The loss is the
full-vocabulary forward KL, computed in row chunks with activation
checkpointing so [rows x V] intermediates stay bounded.
Reference: online-speculation/src/blockspec/parallel/training.py:22-137.
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
    tokens: Tensor        # [B, blocks * K] noisy draft inputs
    positions: Tensor     # [B, blocks * K]
    allowed: Tensor       # [B, 1, blocks * K, T + blocks * K]
    teacher_rows: Tensor  # [B, blocks * (K-1)] clean positions whose AR law teaches
    student_rows: Tensor  # [blocks * (K-1)] draft rows


def sample_anchors(tokens: Tensor, block_size: int, count: int, *, generator=None) -> Tensor:
    if tokens.ndim != 2 or block_size < 2 or count < 1 or tokens.shape[1] < block_size:
        raise ValueError("a nonempty batch, anchors and a complete block are required")
    return torch.randint(tokens.shape[1] - block_size + 1, (tokens.shape[0], count), device=tokens.device,
                         generator=generator)


def anchor_layout(tokens: Tensor, anchors: Tensor, block_size: int, mask_token_id: int) -> AnchorLayout:
    B, T = tokens.shape
    if anchors.ndim != 2 or anchors.shape[0] != B or anchors.dtype != torch.long:
        raise ValueError("integer anchors[batch, blocks] required")
    if ((anchors < 0) | (anchors + block_size > T)).any():
        raise ValueError("each anchor needs a complete block inside the sequence")
    nb = anchors.shape[1]
    pos = anchors[..., None] + torch.arange(block_size, device=tokens.device)           # [B, nb, K]
    noisy = tokens.new_full((B, nb, block_size), mask_token_id)
    noisy[:, :, 0] = tokens.gather(1, anchors)
    total = nb * block_size
    prefix = torch.arange(T, device=tokens.device)[None, None, :] < anchors.repeat_interleave(block_size, 1)[..., None]
    blk = torch.arange(total, device=tokens.device) // block_size
    same = (blk[:, None] == blk[None, :])[None].expand(B, -1, -1)
    allowed = torch.cat((prefix, same), -1)[:, None]
    rows = torch.arange(total, device=tokens.device).view(nb, block_size)[:, :-1].reshape(-1)
    return AnchorLayout(noisy.reshape(B, total), pos.reshape(B, total), allowed, pos[:, :, :-1].reshape(B, -1), rows)


def forward_kl(student_logits: Tensor, teacher_logits: Tensor) -> Tensor:
    lp = teacher_logits.detach().float().log_softmax(-1)
    lq = student_logits.float().log_softmax(-1)
    return (lp.exp() * (lp - lq)).sum(-1).mean()


def distillation_loss(model, tokens: Tensor, anchors: Tensor, *, block_size=None, chunk_rows: int = 32,
                      draft_weights=None) -> Tensor:
    K = model.config.block_size if block_size is None else block_size
    if chunk_rows < 1:
        raise ValueError("positive head chunk size required")
    if any(p.requires_grad for n, p in model.named_parameters() if ".attention.draft." not in n):
        raise ValueError("freeze shared / AR parameters (train_draft_only) before distillation")
    lay = anchor_layout(tokens, anchors, K, model.config.mask_token_id)
    H = model.config.hidden_size
    with torch.no_grad():
        teacher = model(tokens, compute_logits=False)
        th = teacher.hidden.gather(1, lay.teacher_rows[..., None].expand(-1, -1, H)).reshape(-1, H)
    opts = dict(view="draft", cache=teacher.cache, positions=lay.positions, allowed=lay.allowed,
                compute_logits=False)
    student = (model(lay.tokens, **opts) if draft_weights is None
               else torch.func.functional_call(model, draft_weights, (lay.tokens,), opts))
    sh = student.hidden[:, lay.student_rows].reshape(-1, H)
    n = sh.shape[0]

    def chunk(s_rows, t_rows):
        with torch.no_grad():
            tl = F.linear(t_rows, model.head.weight)
        return forward_kl(F.linear(s_rows, model.head.weight), tl)

    terms = [checkpoint(chunk, sh[a:b], th[a:b], use_reentrant=False) * ((b - a) / n)
             for a, b in ((s, min(n, s + chunk_rows)) for s in range(0, n, chunk_rows))]
    return torch.stack(terms).sum()


def distillation_update(model, batches, optimizer, *, learning_rate: float, clip_grad: float = 1.0,
                        chunk_rows: int = 32, autocast=nullcontext, master=None) -> dict:
    """One AdamW step over fixed (tokens, anchors) micro-batches on the draft parameters."""
    if not batches or any(not math.isfinite(v) or v <= 0 for v in (learning_rate, clip_grad)):
        raise ValueError("micro-batches and finite positive optimizer scales required")
    resident = dict(model.named_parameters())
    expected = {n: p for n, p in resident.items() if ".attention.draft." in n}
    selected = expected if master is None else master
    params = [p for g in optimizer.param_groups for p in g["params"]]
    if selected.keys() != expected.keys() or {id(p) for p in params} != {id(p) for p in selected.values()}:
        raise ValueError("the optimizer must own exactly the draft parameter set")
    for g in optimizer.param_groups:
        g["lr"] = learning_rate
    optimizer.zero_grad(set_to_none=True)
    losses = []
    try:
        with torch.enable_grad():
            for tokens, anchors in batches:
                w = None if master is None else {n: p.to(resident[n].dtype) for n, p in master.items()}
                with autocast():
                    loss = distillation_loss(model, tokens, anchors, chunk_rows=chunk_rows, draft_weights=w)
                if not torch.isfinite(loss):
                    raise FloatingPointError("nonfinite distillation loss")
                (loss / len(batches)).backward()
                losses.append(float(loss.detach()))
        norm = torch.nn.utils.clip_grad_norm_(params, clip_grad, error_if_nonfinite=True)
        optimizer.step()
    finally:
        optimizer.zero_grad(set_to_none=True)
    return {"loss": sum(losses) / len(losses), "learning_rate": learning_rate, "gradient_norm": float(norm)}
