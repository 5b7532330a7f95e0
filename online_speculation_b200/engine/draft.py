"""Block-bidirectional draft head and its online learner.

Draft head: one decoder layer whose *attention* has its own projections (the
draft view) while it shares the norms, MLP, final norm and output head of the
target's last layer.  A block ``[anchor, MASK x (K-1)]`` is embedded, attends
bidirectionally within the block and read-only to the target's last-layer KV
history (KV-history reuse), and the head produces proposal logits for the
K - 1 positions after the anchor.  This is the shared-backbone dual-view
drafting of online-speculation/src/blockspec/parallel/backbone.py:86-148 and
branches.py:27-52, restricted to a one-layer suffix so a draft costs one layer
plus the head.

Online learner (online-speculation/src/blockspec/parallel/online.py:44-196):
fp32 master copies of the draft attention weights; feedback blocks keep the
teacher (target verify) logits of the reached rows; every ``stride`` verified
blocks the learner replays the latest ``replay_blocks`` rounds, minimises
full-vocabulary TV or forward KL to the teacher, clips the global gradient
norm, takes a fused AdamW step (sm_100a kernel) and publishes bf16 execution
weights in place between rounds.
"""

from __future__ import annotations

import copy
import hashlib
import math
import time
from collections import deque
from dataclasses import asdict, dataclass

import torch
import torch.nn.functional as F

from ..models.decoder import DecoderWeights
from ..ops import kernels as K
from .runner import ModelRunner, StepMeta


@dataclass
class DraftWeights:
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor | None
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    w_o: torch.Tensor

    FIELDS = ("w_qkv", "b_qkv", "q_norm", "k_norm", "w_o")

    def tensors(self) -> dict[str, torch.Tensor]:
        """Named draft tensors (views into one flat bf16 buffer), in storage order."""
        return {k: getattr(self, k) for k in self.FIELDS if getattr(self, k) is not None}


def init_draft(weights: DecoderWeights, *, seed: int = 1, std: float = 0.02, copy_from_target: bool = False
               ) -> DraftWeights:
    """Random-init (or copy the last layer's AR projections into) the draft view.

    The flat bf16 storage lets the learner publish all draft tensors with one
    fused AdamW launch.
    """
    lw = weights.layers[-1]
    parts = [("w_qkv", lw.w_qkv), ("b_qkv", lw.b_qkv), ("q_norm", lw.q_norm), ("k_norm", lw.k_norm), ("w_o", lw.w_o)]
    total = sum(t.numel() for _, t in parts if t is not None)
    flat = torch.empty(total, dtype=torch.bfloat16, device=weights.device)
    g = torch.Generator(device=weights.device).manual_seed(seed)
    views = {}
    off = 0
    for name, t in parts:
        if t is None:
            views[name] = None
            continue
        v = flat[off:off + t.numel()].view_as(t)
        off += t.numel()
        if copy_from_target or name in ("q_norm", "k_norm"):
            v.copy_(t)
        elif name == "b_qkv":
            v.zero_()
        else:
            v.copy_((torch.randn(t.shape, generator=g, device=t.device) * std).to(torch.bfloat16))
            if name == "w_o" or name == "w_qkv":
                # keep padded (zero) head slots at zero
                v.mul_((t != 0).any(dim=1 if name == "w_qkv" else 0, keepdim=True))
        views[name] = v
    dw = DraftWeights(**views)
    dw.flat = flat
    return dw


class DraftHead:
    def __init__(self, runner: ModelRunner, draft: DraftWeights, *, block_size: int = 4, mask_token_id: int | None = None):
        if block_size < 2:
            raise ValueError("block drafting needs block_size >= 2")
        self.runner = runner
        self.draft = draft
        self.block_size = block_size
        cfg = runner.cfg
        self.mask_token_id = cfg.vocab_size - 1 if mask_token_id is None else mask_token_id
        self.layer = cfg.num_hidden_layers - 1

    def forward(self, meta: StepMeta, logit_rows: torch.Tensor) -> torch.Tensor:
        """meta: ids = [anchor, MASK...] per block, bidirectional plan over history + block.
        Writes the draft K/V of the block into the last layer's cache slots (the
        verify pass overwrites them).  Returns fp32 logits of ``logit_rows``."""
        r = self.runner
        eps = r.cfg.rms_norm_eps
        T = meta.ids.numel()
        lw = r.w.layers[self.layer]
        h = r._buf("dh", (T, r.cfg.hidden_size))
        r.embed(meta.ids, h)
        x = r._buf("dx", (T, r.cfg.hidden_size))
        K.rmsnorm(h, lw.in_norm, eps, out=x)
        d = self.draft
        pend = r.attention_block(self.layer, x, meta, wq=d.w_qkv, bias=d.b_qkv, q_norm=d.q_norm, k_norm=d.k_norm,
                                 wo=d.w_o, residual=h)
        if r.comm.world == 1:
            K.rmsnorm(h, lw.post_norm, eps, out=x)
        else:
            K.rmsnorm(h, lw.post_norm, eps, out=x, residual=h, delta=pend)
        pend = r.mlp_block(self.layer, x, residual=h)
        if r.comm.world == 1:
            return r.logits(h, logit_rows)
        K.rmsnorm(h, r.w.final_norm, eps, out=x, residual=h, delta=pend)
        sel = r._index_rows(x, logit_rows)
        return r.logits(sel, None, normed=True)


# ------------------------------------------------------------------ learner --
class _ReduceFromTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        import torch.distributed as dist

        y = x.clone()
        dist.all_reduce(y, group=group)
        return y

    @staticmethod
    def backward(ctx, g):
        return g, None


class _CopyToTP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x

    @staticmethod
    def backward(ctx, g):
        import torch.distributed as dist

        g = g.clone()
        dist.all_reduce(g, group=ctx.group)
        return g, None


def _reduce(x, comm):
    return x if comm.world == 1 else _ReduceFromTP.apply(x, comm.group)


def _copy(x, comm):
    return x if comm.world == 1 else _CopyToTP.apply(x, comm.group)


@dataclass(frozen=True)
class SuffixConfig:
    """Online learner policy (field names follow the reference SuffixConfig)."""

    last_layers: int = 1
    stride: int = 64          # verified blocks between updates
    replay_blocks: int = 1    # rounds of feedback replayed per update
    learning_rate: float = 1e-5
    clip_norm: float = 1.0
    loss: str = "tv"

    def __post_init__(self):
        if self.last_layers != 1:
            raise ValueError("the draft head is a one-layer suffix")
        if self.stride < 1 or self.replay_blocks < 1:
            raise ValueError("positive stride and replay window required")
        if not (math.isfinite(self.learning_rate) and self.learning_rate > 0 and self.clip_norm > 0):
            raise ValueError("positive learning rate and clip norm required")
        if self.loss not in ("tv", "forward_kl"):
            raise ValueError("loss must be tv or forward_kl")


@dataclass
class FeedbackRound:
    """One verified round of a batch of blocks (device tensors, detached)."""

    block_ids: torch.Tensor      # [B, K] draft inputs
    positions: torch.Tensor      # [B, K]
    hist_pages: list[list[int]]  # page ids of each block's history (last layer)
    hist_len: list[int]
    teacher: torch.Tensor        # [B, K-1, V] fp32 target logits (local vocab shard)
    valid: torch.Tensor          # [B] reached rows (0..K-1)


class SuffixLearner:
    def __init__(self, head: DraftHead, config: SuffixConfig = SuffixConfig()):
        self.head = head
        self.config = config
        d = head.draft
        self.names = [n for n, t in d.tensors().items()]
        self.master = d.flat.float().clone()
        self.grad = torch.zeros_like(self.master)
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.norm_buf = torch.zeros(1, dtype=torch.float32, device=self.master.device)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=self.master.device)
        self.replay: deque[FeedbackRound] = deque(maxlen=config.replay_blocks)
        self.blocks_seen = 0
        self.updates = 0
        self.update_seconds = 0.0
        self.last_loss: float | None = None
        self.step = 0
        self.frozen_fingerprint = self._fingerprint()

    def _fingerprint(self) -> str:
        w = self.head.runner.w
        h = hashlib.sha256()
        lw = w.layers[-1]
        for t in (lw.w_gu, lw.w_down, lw.post_norm, lw.in_norm, w.final_norm):
            h.update(t.detach().flatten()[:4096].float().cpu().numpy().tobytes())
        return h.hexdigest()

    def _views(self, flat: torch.Tensor) -> dict[str, torch.Tensor]:
        out, off = {}, 0
        for n, t in self.head.draft.tensors().items():
            out[n] = flat[off:off + t.numel()].view_as(t)
            off += t.numel()
        return out

    def observe(self, fb: FeedbackRound) -> dict | None:
        self.replay.append(fb)
        before = self.blocks_seen // self.config.stride
        self.blocks_seen += fb.block_ids.shape[0]
        if self.blocks_seen // self.config.stride > before:
            return self.update()
        return None

    def _forward_loss(self, fb: FeedbackRound, params: dict[str, torch.Tensor]) -> torch.Tensor:
        r = self.head.runner
        cfg = r.cfg
        comm = r.comm
        lw = r.w.layers[-1]
        kc, vc = r.cache.layer(cfg.num_hidden_layers - 1)
        B, Kb = fb.block_ids.shape
        D, H = 128, cfg.hidden_size
        eps = cfg.rms_norm_eps
        emb = r.w.embed[fb.block_ids.long()].float()                      # [B, K, H]

        def norm(x, w):
            return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w.float()

        x = _copy(norm(emb, lw.in_norm), comm)
        qkv = x @ params["w_qkv"].t()
        if "b_qkv" in params:
            qkv = qkv + params["b_qkv"]
        qs, ks = r.q_slots, r.kv_slots
        q = qkv[..., : qs * D].view(B, Kb, qs, D)
        k = qkv[..., qs * D:(qs + ks) * D].view(B, Kb, ks, D)
        v = qkv[..., (qs + ks) * D:(qs + 2 * ks) * D].view(B, Kb, ks, D)
        if "q_norm" in params:
            q = norm(q, params["q_norm"])
            k = norm(k, params["k_norm"])
        inv = r.w.inv_freq
        ang = fb.positions.float()[..., None] * inv                          # [B, K, D/2]
        cos, sin = ang.cos()[:, :, None], ang.sin()[:, :, None]

        def rope(t):
            a, b = t[..., : D // 2], t[..., D // 2:]
            return torch.cat((a * cos - b * sin, b * cos + a * sin), -1)

        q, k = rope(q), rope(k)
        Lmax = max(fb.hist_len) if fb.hist_len else 0
        G = qs // ks
        pages_needed = -(-Lmax // 32) if Lmax else 0
        if pages_needed:
            table = torch.tensor([p[:pages_needed] + [0] * (pages_needed - len(p[:pages_needed])) for p in fb.hist_pages],
                                 dtype=torch.long, device=emb.device)
            hk = kc[table].permute(0, 2, 1, 3, 4).reshape(B, ks, pages_needed * 32, D)[:, :, :Lmax].float()
            hv = vc[table].permute(0, 2, 1, 3, 4).reshape(B, ks, pages_needed * 32, D)[:, :, :Lmax].float()
        else:
            hk = hv = torch.zeros(B, ks, 0, D, device=emb.device)
        kk = torch.cat((hk, k.permute(0, 2, 1, 3)), 2)                      # [B, ks, L+K, D]
        vv = torch.cat((hv, v.permute(0, 2, 1, 3)), 2)
        qq = q.permute(0, 2, 1, 3).reshape(B, ks, G, Kb, D).reshape(B, ks, G * Kb, D)
        scores = qq @ kk.transpose(-1, -2) / math.sqrt(D)                   # [B, ks, G*K, L+K]
        hl = torch.tensor(fb.hist_len, device=emb.device)
        key = torch.arange(Lmax + Kb, device=emb.device)
        visible = (key[None, :] < hl[:, None]) | (key[None, :] >= Lmax)      # history (ragged) + block
        scores = scores.masked_fill(~visible[:, None, None, :], float("-inf"))
        att = (scores.softmax(-1) @ vv).view(B, ks, G, Kb, D).permute(0, 3, 1, 2, 4).reshape(B, Kb, qs * D)
        h = emb + _reduce(att @ params["w_o"].t(), comm)
        x2 = _copy(norm(h, lw.post_norm), comm)
        gu = (x2.to(torch.bfloat16) @ lw.w_gu.t()).float()
        gu = gu.view(B, Kb, -1, 2, 64)
        act = (F.silu(gu[..., 0, :]) * gu[..., 1, :]).reshape(B, Kb, -1)
        h = h + _reduce((act.to(torch.bfloat16) @ lw.w_down.t()).float(), comm)
        y = _copy(norm(h[:, : Kb - 1], r.w.final_norm), comm)
        logits = (y.to(torch.bfloat16) @ r.w.head.t()).float()              # [B, K-1, V_local]
        rows = torch.arange(Kb - 1, device=emb.device)[None, :] < fb.valid[:, None]
        return self._divergence(logits[rows], fb.teacher[rows], comm), int(rows.sum())

    def _divergence(self, student: torch.Tensor, teacher: torch.Tensor, comm) -> torch.Tensor:
        """Sum over rows of TV or KL(teacher || student) over the (possibly sharded) vocabulary."""
        def lse(z):
            m = z.max(-1, keepdim=True).values.detach()
            if comm.world > 1:
                import torch.distributed as dist

                dist.all_reduce(m, op=dist.ReduceOp.MAX, group=comm.group)
            s = _reduce((z - m).exp().sum(-1, keepdim=True), comm)
            return m + s.log()

        log_q = student - lse(student)
        with torch.no_grad():
            log_p = teacher - lse(teacher)
        if self.config.loss == "tv":
            per = 0.5 * (log_q.exp() - log_p.exp()).abs().sum(-1)
        else:
            per = (log_p.exp() * (log_p - log_q)).sum(-1)
        return _reduce(per.sum(), comm)

    def update(self) -> dict | None:
        if not self.replay:
            return None
        dev = self.master.device
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        start = time.perf_counter()
        params = {n: t.detach().clone().requires_grad_(True) for n, t in self._views(self.master).items()}
        total = 0.0
        rows = sum(int(fb.valid.sum()) for fb in self.replay)
        grads = {n: torch.zeros_like(p) for n, p in params.items()}
        for fb in self.replay:
            loss, _ = self._forward_loss(fb, params)
            loss = loss / max(rows, 1)
            if not torch.isfinite(loss):
                raise FloatingPointError("nonfinite online suffix loss")
            g = torch.autograd.grad(loss, list(params.values()))
            for n, gi in zip(params, g):
                grads[n] += gi
            total += float(loss.detach())
        flat_g = self._views(self.grad)
        for n in params:
            flat_g[n].copy_(grads[n])
        self.step += 1
        K.adamw_step(self.master, self.grad, self.exp_avg, self.exp_avg_sq, step=self.step,
                     lr=self.config.learning_rate, weight_decay=0.0, clip=self.config.clip_norm,
                     publish=self.head.draft.flat, norm_out=self.norm_buf, nonfinite=self.nonfinite)
        if dev.type == "cuda":
            torch.cuda.synchronize(dev)
        elapsed = time.perf_counter() - start
        self.updates += 1
        self.update_seconds += elapsed
        self.last_loss = total
        self.replay.clear()
        return {"loss": total, "gradient_norm": float(self.norm_buf.sqrt()), "seconds": elapsed,
                "version": self.updates}

    # ---- checkpoint (format "blockspec-dual-suffix-v1" fields) ----
    def state_dict(self) -> dict:
        if self.replay:
            raise ValueError("save online state at a request boundary after clearing replay")
        return {"format": "blockspec-dual-suffix-v1", "config": asdict(self.config),
                "model_config": self.head.runner.cfg.to_dict(), "frozen_fingerprint": self.frozen_fingerprint,
                "master": self.master.cpu().clone(),
                "optimizer": {"exp_avg": self.exp_avg.cpu().clone(), "exp_avg_sq": self.exp_avg_sq.cpu().clone(),
                              "step": self.step},
                "rounds": self.blocks_seen, "updates": self.updates, "version": self.updates,
                "update_seconds": self.update_seconds, "last_loss": self.last_loss}

    def load_state_dict(self, state: dict) -> None:
        if (state.get("format") != "blockspec-dual-suffix-v1" or state.get("config") != asdict(self.config)
                or state.get("model_config") != self.head.runner.cfg.to_dict()
                or state.get("frozen_fingerprint") != self.frozen_fingerprint):
            raise ValueError("online state must match its model, update policy and frozen weights")
        master = state["master"]
        if master.shape != self.master.shape or master.dtype != torch.float32 or not torch.isfinite(master).all():
            raise ValueError("finite FP32 suffix masters of matching shape required")
        self.master.copy_(master)
        self.exp_avg.copy_(state["optimizer"]["exp_avg"])
        self.exp_avg_sq.copy_(state["optimizer"]["exp_avg_sq"])
        self.step = int(state["optimizer"]["step"])
        self.blocks_seen = int(state["rounds"])
        self.updates = int(state["updates"])
        self.update_seconds = float(state["update_seconds"])
        self.last_loss = state["last_loss"]
        self.head.draft.flat.copy_(self.master)
        self.replay.clear()
