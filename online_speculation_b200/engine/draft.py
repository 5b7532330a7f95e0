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

    def forward(self, meta: StepMeta, logit_rows: torch.Tensor, *, gather: bool = True) -> torch.Tensor:
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
        part = r.attention_block(self.layer, x, meta, wq=d.w_qkv, bias=d.b_qkv, q_norm=d.q_norm, k_norm=d.k_norm,
                                 wo=d.w_o, residual=h)
        if r.comm.world == 1:
            K.rmsnorm(h, lw.post_norm, eps, out=x)
        else:
            r.comm.reduce_add_norm(part, h, lw.post_norm, x, eps)
        part = r.mlp_block(self.layer, x, residual=h)
        if r.comm.world == 1:
            return r.logits(h, logit_rows)
        r.comm.reduce_add_norm(part, h, r.w.final_norm, x, eps)
        sel = r._index_rows(x, logit_rows)
        return r.logits(sel, None, normed=True, gather=gather)


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
    """One verified round of a batch of blocks, as device tensors.

    When the round comes from a captured round graph these are that graph's
    static buffers, read in place right after the round (before the next one
    overwrites them), so the learner update can itself be a replayed graph.
    """

    block_ids: torch.Tensor      # [B, K] int32 draft inputs [anchor, MASK...]
    positions: torch.Tensor      # [B, K] int32 absolute positions of the block
    table: torch.Tensor          # [B, max_pages] int32 page table (history = keys < positions[:, 0])
    teacher: torch.Tensor        # [B * K, V_local] fp32 target verify logits
    count: torch.Tensor          # [B] int32 accepted draft tokens of the round
    active: torch.Tensor         # [B] fp32, 1 for real blocks, 0 for padding rows
    blocks: int                  # number of real blocks


class _PublishedMM(torch.autograd.Function):
    """x @ W^T in bf16 with an fp32 result, W an fp32 master leaf whose bf16 copy is
    already published (the fused AdamW writes bf16(master) after every step).

    Same numerics as ``(x.bf16() @ W.bf16().T).float()`` under autograd, without
    converting the master to bf16 in the forward or the bf16 weight gradient
    through a separate cast kernel in the backward.
    """

    @staticmethod
    def forward(ctx, x, w_master, w_pub):
        xb = x.to(torch.bfloat16)
        ctx.save_for_backward(xb, w_pub)
        return (xb @ w_pub.t()).float()

    @staticmethod
    def backward(ctx, g):
        xb, w_pub = ctx.saved_tensors
        gb = g.to(torch.bfloat16)
        gx = (gb @ w_pub).float()
        gw = (gb.reshape(-1, gb.shape[-1]).t() @ xb.reshape(-1, xb.shape[-1])).float()
        return gx, gw, None


class SuffixLearner:
    """Online suffix learner of the draft attention (fp32 masters, fused AdamW)."""

    def __init__(self, head: DraftHead, config: SuffixConfig = SuffixConfig(), *, use_graphs: bool = True):
        self.head = head
        self.config = config
        d = head.draft
        dev = d.flat.device
        self.master = torch.nn.Parameter(d.flat.float().clone())
        self.exp_avg = torch.zeros_like(self.master, requires_grad=False)
        self.exp_avg_sq = torch.zeros_like(self.master, requires_grad=False)
        # one autograd leaf per draft tensor, aliasing the flat master's storage: the backward then
        # yields one gradient per tensor (no zero-filled master-sized accumulator and scatter-add),
        # gathered once into the flat gradient buffer the fused AdamW reads
        self.leaves = {n: t.detach().requires_grad_(True) for n, t in self._views(self.master.data).items()}
        self.grad_buf = torch.zeros_like(self.master, requires_grad=False)
        self.norm_buf = torch.zeros(1, dtype=torch.float32, device=dev)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=dev)
        self.step_t = torch.zeros(1, dtype=torch.int32, device=dev)
        self.loss_buf = torch.zeros(1, dtype=torch.float32, device=dev)
        self.use_graphs = use_graphs and dev.type == "cuda"
        self._graphs: dict[tuple, torch.cuda.CUDAGraph] = {}
        self.blocks_seen = 0
        self.updates = 0
        self.update_seconds = 0.0
        self.step = 0
        self.frozen_fingerprint = self._fingerprint()

    @property
    def last_loss(self) -> float:
        return float(self.loss_buf)

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

    def observe(self, fb: FeedbackRound) -> bool:
        """Record one verified round; runs an update every ``stride`` verified blocks."""
        before = self.blocks_seen // self.config.stride
        self.blocks_seen += fb.blocks
        if self.blocks_seen // self.config.stride > before:
            self.update(fb)
            return True
        return False

    # ---- replayed suffix forward + loss (static shapes, no host syncs) ----
    def _loss(self, fb: FeedbackRound) -> torch.Tensor:
        r = self.head.runner
        cfg = r.cfg
        comm = r.comm
        lw = r.w.layers[-1]
        kc, vc = r.cache.layer(cfg.num_hidden_layers - 1)
        B, Kb = fb.block_ids.shape
        D = 128
        eps = cfg.rms_norm_eps
        params = self.leaves
        bf = torch.bfloat16

        def norm(x, w):
            return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w.float()

        def mm(x, w):  # bf16 tensor-core matmul with fp32 result
            return (x.to(bf) @ w.to(bf).t()).float()

        published = self.head.draft.tensors()    # bf16(master), written by every AdamW step

        emb = r.w.embed[fb.block_ids.long()].float()                        # [B, K, H]
        x = _copy(norm(emb, lw.in_norm), comm)
        qkv = _PublishedMM.apply(x, params["w_qkv"], published["w_qkv"])
        if "b_qkv" in params:
            qkv = qkv + params["b_qkv"]
        qs, ks = r.q_slots, r.kv_slots
        G = qs // ks
        q = qkv[..., : qs * D].view(B, Kb, qs, D)
        k = qkv[..., qs * D:(qs + ks) * D].view(B, Kb, ks, D)
        v = qkv[..., (qs + ks) * D:(qs + 2 * ks) * D].view(B, Kb, ks, D)
        if "q_norm" in params:
            q = norm(q, params["q_norm"])
            k = norm(k, params["k_norm"])
        ang = fb.positions.float()[..., None] * r.w.inv_freq                # [B, K, D/2]
        cos, sin = ang.cos()[:, :, None], ang.sin()[:, :, None]

        def rope(t):
            a, b = t[..., : D // 2], t[..., D // 2:]
            return torch.cat((a * cos - b * sin, b * cos + a * sin), -1)

        q, k = rope(q), rope(k)
        att = self._draft_attention(q, k, v, fb, kc, vc)                    # [B, K, qs * D]
        h = emb + _reduce(_PublishedMM.apply(att, params["w_o"], published["w_o"]), comm)
        x2 = _copy(norm(h, lw.post_norm), comm)
        gu = mm(x2, lw.w_gu).view(B, Kb, -1, 2, 64)
        act = (F.silu(gu[..., 0, :]) * gu[..., 1, :]).reshape(B, Kb, -1)
        h = h + _reduce(mm(act, lw.w_down), comm)
        y = _copy(norm(h[:, : Kb - 1], r.w.final_norm), comm)                # [B, K-1, H]
        teacher = fb.teacher.view(B, Kb, -1)[:, : Kb - 1].reshape(B * (Kb - 1), -1)
        per = K.head_divergence(y.reshape(B * (Kb - 1), -1), r.w.head, teacher, self.config.loss,
                                comm if comm.world > 1 else None).view(B, Kb - 1)
        valid = torch.minimum(fb.count + 1, torch.full_like(fb.count, Kb - 1))
        w = (torch.arange(Kb - 1, device=emb.device)[None, :] < valid[:, None]).float() * fb.active[:, None]
        return (per * w).sum() / w.sum().clamp_min(1.0)

    @staticmethod
    def _draft_attention(q, k, v, fb: FeedbackRound, kc, vc) -> torch.Tensor:
        """Block queries over the frozen paged history (keys before the block) plus the block itself.

        History scores use a bf16 tensor-core matmul with fp32 softmax; only the
        block's q, k and v carry gradients.  (A fused masked SDPA was measured on
        B200 at 1.1 ms forward + backward for 64 blocks x 1088 keys, about twice
        this explicit form.)  Returns fp32 [B, K, qs * D].
        """
        B, Kb, qs, D = q.shape
        ks = k.shape[2]
        G = qs // ks
        P = fb.table.shape[1]
        L = P * kc.shape[2]
        bf = torch.bfloat16
        # one gather of the history pages straight into [B, ks, L, D]: cache row (page * ks + head) holds
        # that head's 32 keys of the page
        page = kc.shape[2]
        idx = (fb.table.long()[:, None, :] * ks + torch.arange(ks, device=q.device)[None, :, None]).reshape(-1)
        hk = kc.view(-1, page * D).index_select(0, idx).view(B, ks, L, D)   # bf16 (frozen)
        hv = vc.view(-1, page * D).index_select(0, idx).view(B, ks, L, D)
        qq = q.permute(0, 2, 1, 3).reshape(B, ks, G * Kb, D)               # [B, ks, G*K, D]
        kb = k.permute(0, 2, 1, 3)                                         # [B, ks, K, D]
        vb = v.permute(0, 2, 1, 3)
        scale = D ** -0.5
        s_hist = (qq.to(bf) @ hk.transpose(-1, -2)).float() * scale         # [B, ks, G*K, L]
        s_blk = (qq @ kb.transpose(-1, -2)) * scale                         # [B, ks, G*K, K]
        key = torch.arange(L, device=q.device)
        visible = key[None, :] < fb.positions[:, :1]                         # [B, L] history keys
        s_hist = s_hist.masked_fill(~visible[:, None, None, :], float("-inf"))
        prob = torch.cat((s_hist, s_blk), -1).softmax(-1)
        att = (prob[..., :L].to(bf) @ hv).float() + prob[..., L:] @ vb
        return att.view(B, ks, G, Kb, D).permute(0, 3, 1, 2, 4).reshape(B, Kb, qs * D)

    def _divergence(self, student: torch.Tensor, teacher: torch.Tensor, comm) -> torch.Tensor:
        """Per-row TV or KL(teacher || student) over the (possibly vocabulary-sharded) rows."""
        def lse(z):
            m = z.max(-1, keepdim=True).values.detach()
            if comm.world > 1:
                import torch.distributed as dist

                dist.all_reduce(m, op=dist.ReduceOp.MAX, group=comm.group)
            return m + _reduce((z - m).exp().sum(-1, keepdim=True), comm).log()

        log_q = student - lse(student)
        with torch.no_grad():
            log_p = teacher - lse(teacher)
        if self.config.loss == "tv":
            per = 0.5 * (log_q.exp() - log_p.exp()).abs().sum(-1)
        else:
            per = (log_p.exp() * (log_p - log_q)).sum(-1)
        return _reduce(per, comm)

    def _step(self, fb: FeedbackRound) -> None:
        loss = self._loss(fb)
        leaves = list(self.leaves.values())
        grads = torch.autograd.grad(loss, leaves, allow_unused=True)
        torch.cat([(g if g is not None else torch.zeros_like(t)).reshape(-1) for g, t in zip(grads, leaves)],
                  out=self.grad_buf)
        grad = self.grad_buf
        self.loss_buf.copy_(loss.detach())
        self.step_t.add_(1)
        K.adamw_step(self.master.data, grad, self.exp_avg, self.exp_avg_sq, step=1, lr=self.config.learning_rate,
                     weight_decay=0.0, clip=self.config.clip_norm, publish=self.head.draft.flat,
                     norm_out=self.norm_buf, nonfinite=self.nonfinite, step_tensor=self.step_t)

    def update(self, fb: FeedbackRound) -> None:
        dev = self.master.device
        start = time.perf_counter()
        if self.use_graphs:
            key = (fb.block_ids.data_ptr(), fb.teacher.data_ptr(), tuple(fb.block_ids.shape))
            g = self._graphs.get(key)
            if g is None:
                g = self._capture(fb)
                self._graphs[key] = g
            g.replay()
        else:
            self._step(fb)
        self.step += 1
        self.updates += 1
        self.update_seconds += time.perf_counter() - start

    def _capture(self, fb: FeedbackRound) -> "torch.cuda.CUDAGraph":
        # warm up autograd on a side stream without changing the optimizer state
        saved = [t.clone() for t in (self.master.data, self.exp_avg, self.exp_avg_sq, self.step_t,
                                     self.head.draft.flat)]
        s = torch.cuda.Stream(device=self.master.device)
        s.wait_stream(torch.cuda.current_stream(self.master.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step(fb)
        torch.cuda.current_stream(self.master.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._step(fb)
        for t, v in zip((self.master.data, self.exp_avg, self.exp_avg_sq, self.step_t, self.head.draft.flat), saved):
            t.copy_(v)
        return g

    def close(self) -> None:
        """Drop captured update graphs (call before destroying a process group)."""
        self._graphs.clear()

    def check_finite(self) -> None:
        if int(self.nonfinite.item()):
            self.nonfinite.zero_()
            raise FloatingPointError("nonfinite online suffix gradient; the step was skipped")

    # ---- checkpoint (format "blockspec-dual-suffix-v1" fields) ----
    def state_dict(self) -> dict:
        self.check_finite()
        return {"format": "blockspec-dual-suffix-v1", "config": asdict(self.config),
                "model_config": self.head.runner.cfg.to_dict(), "frozen_fingerprint": self.frozen_fingerprint,
                "master": self.master.detach().cpu().clone(),
                "optimizer": {"exp_avg": self.exp_avg.cpu().clone(), "exp_avg_sq": self.exp_avg_sq.cpu().clone(),
                              "step": int(self.step_t.item())},
                "rounds": self.blocks_seen, "updates": self.updates, "version": self.updates,
                "update_seconds": self.update_seconds, "last_loss": self.last_loss if self.updates else None}

    def load_state_dict(self, state: dict) -> None:
        if (state.get("format") != "blockspec-dual-suffix-v1" or state.get("config") != asdict(self.config)
                or state.get("model_config") != self.head.runner.cfg.to_dict()
                or state.get("frozen_fingerprint") != self.frozen_fingerprint):
            raise ValueError("online state must match its model, update policy and frozen weights")
        master = state["master"]
        if master.shape != self.master.shape or master.dtype != torch.float32 or not torch.isfinite(master).all():
            raise ValueError("finite FP32 suffix masters of matching shape required")
        with torch.no_grad():
            self.master.copy_(master)
        self.exp_avg.copy_(state["optimizer"]["exp_avg"])
        self.exp_avg_sq.copy_(state["optimizer"]["exp_avg_sq"])
        self.step = int(state["optimizer"]["step"])
        self.step_t.fill_(self.step)
        self.blocks_seen = int(state["rounds"])
        self.updates = int(state["updates"])
        self.update_seconds = float(state["update_seconds"])
        if state["last_loss"] is not None:
            self.loss_buf.fill_(float(state["last_loss"]))
        self.head.draft.flat.copy_(self.master.detach())
