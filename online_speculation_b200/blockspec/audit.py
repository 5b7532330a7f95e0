"""Same-prefix audit of a learned draft suffix against the original
(online-speculation/src/blockspec/parallel/audit.py).

For held-out sequences, random anchors produce draft blocks; the AR teacher
law at each drafted position is compared with both the original and the
learned draft laws (KL and TV), so an online update can be checked on
identical inputs.
"""

from __future__ import annotations

import torch

from .model import DualViewDecoder
from .online import divergence
from .training import anchor_layout


@torch.no_grad()
def audit(original: DualViewDecoder, learned: DualViewDecoder, sequences: torch.Tensor, anchors: torch.Tensor) -> dict:
    K = original.config.block_size
    lay = anchor_layout(sequences, anchors, K, original.config.mask_token_id)
    out = {}
    for name, model in (("original", original), ("learned", learned)):
        teacher = model(sequences)
        tl = teacher.logits.gather(1, lay.teacher_rows[..., None].expand(-1, -1, teacher.logits.shape[-1]))
        student = model(lay.tokens, view="draft", cache=teacher.cache, positions=lay.positions, allowed=lay.allowed)
        sl = student.logits[:, lay.student_rows]
        out[name] = {"kl": float(divergence(sl, tl, "forward_kl").mean()),
                     "tv": float(divergence(sl, tl, "tv").mean())}
    out["kl_change"] = out["learned"]["kl"] - out["original"]["kl"]
    out["tv_change"] = out["learned"]["tv"] - out["original"]["tv"]
    return out
