"""Differentiable MoE FFN over frozen expert weights (gradients flow to the input and the router input).

Forward: the kernel path of ``ops.kernels.moe_ffn`` with the gate / up GEMM
kept unfused so the SwiGLU inputs can be saved.  Backward, per layer:

* combine:   d y_slot = w_tj d h_t,   d w_tj = <d h_t, y_slot>
* down:      d act = d y W_down_e          (grouped GEMM on pre-transposed W_down)
* SwiGLU:    d g = d act u silu'(g),  d u = d act silu(g)
* gate / up: d xp = d gu W_gu_e            (grouped GEMM on pre-transposed W_gu)
* dispatch:  d x_t = sum_j d xp_slot(t, j)
* router:    d logits = p (d p - <d p, p>) with d p non-zero on the chosen experts;
             d x += d logits R
All GEMMs are the tcgen05 kernel; the transposed expert weights are built
once per layer (the weights are frozen).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import kernels as K


class FrozenExperts:
    """Expert weights of one layer plus the transposed copies the backward needs."""

    def __init__(self, router: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor, top_k: int, renorm: bool):
        self.router, self.w_gu, self.w_down = router, w_gu, w_down
        self.E = router.shape[0]
        self.H = router.shape[1]
        self.F = w_down.shape[1]
        self.k, self.renorm = top_k, renorm
        E, H, Fd = self.E, self.H, self.F
        self.w_down_t = w_down.view(E, H, Fd).transpose(1, 2).reshape(E * Fd, H).contiguous()   # [E F, H]
        self.w_gu_t = w_gu.view(E, 2 * Fd, H).transpose(1, 2).reshape(E * H, 2 * Fd).contiguous()  # [E H, 2F]
        self.router_t = router.t().contiguous()


def _swiglu_split(gu: torch.Tensor):
    """Interleaved [rows, 2F] tiles of [64 gate | 64 up] -> (gate, up) views [rows, F/64, 64]."""
    t = gu.view(gu.shape[0], -1, 2, 64)
    return t[:, :, 0], t[:, :, 1]


class _MoEFFN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, h, anchor, ex: FrozenExperts):
        ext = K._ext.require()
        T = x.shape[0]
        k, E = ex.k, ex.E
        dev = x.device
        rows = T * k
        xb = x.to(torch.bfloat16).contiguous()
        logits = K.linear(xb, ex.router, out_dtype=torch.float32)
        idx = torch.empty(rows, dtype=torch.int32, device=dev)
        w = torch.empty(rows, dtype=torch.float32, device=dev)
        counts = torch.zeros(E, dtype=torch.int32, device=dev)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        cursor = torch.empty(E, dtype=torch.int32, device=dev)
        slot_of = torch.empty(rows, dtype=torch.int32, device=dev)
        ext.moe_route(logits, k, ex.renorm, idx, w, counts)
        ext.moe_offsets(counts, offsets, cursor)
        xp = torch.empty(rows, ex.H, dtype=torch.bfloat16, device=dev)
        ext.moe_dispatch(xb, idx, cursor, xp, slot_of)
        bn = K.moe_pick_bn(rows, E)
        ws, ctr, st = K.workspace.gemm_workspace(dev), K.workspace.gemm_counters(dev), K.workspace.status(dev)

        def grouped(wt, inp, m_rows, cols, epilogue=0):
            tiles_m = m_rows // 128
            tiles = torch.empty(tiles_m * (-(-rows // 32) + E) * 4, dtype=torch.int32, device=dev)
            total = torch.empty(1, dtype=torch.int32, device=dev)
            ext.grouped_tiles(offsets, E, tiles_m, bn, tiles, total)
            out = torch.empty(rows, cols, dtype=torch.bfloat16, device=dev)
            ext.grouped_gemm(wt, inp, out, epilogue, tiles, total, E, bn, ws, ctr, st)
            return out

        gu = grouped(ex.w_gu, xp, 2 * ex.F, 2 * ex.F)
        g, u = _swiglu_split(gu)
        act = (F.silu(g.float()) * u.float()).to(torch.bfloat16).reshape(rows, ex.F)
        y = grouped(ex.w_down, act, ex.H, ex.H)
        out = h.to(torch.bfloat16).clone()
        ext.moe_combine(y, slot_of, w, out, True)
        ctx.save_for_backward(logits, idx, w, slot_of, offsets, gu, y)
        ctx.ex, ctx.grouped, ctx.rows = ex, grouped, rows
        return out

    @staticmethod
    def backward(ctx, gout):
        logits, idx, w, slot_of, offsets, gu, y = ctx.saved_tensors
        ex, grouped, rows = ctx.ex, ctx.grouped, ctx.rows
        T = gout.shape[0]
        k = ex.k
        g32 = gout.float()
        slots = slot_of.long()
        tok = torch.arange(T, device=gout.device).repeat_interleave(k)
        # combine backward
        dy = torch.empty(rows, ex.H, dtype=torch.bfloat16, device=gout.device)
        dy[slots] = (w[:, None] * g32[tok]).to(torch.bfloat16)
        dw = (g32[tok] * y[slots].float()).sum(-1).view(T, k)
        # down backward
        d_act = grouped(ex.w_down_t, dy, ex.F, ex.F).float()
        gate, up = _swiglu_split(gu)
        gf, uf = gate.float().reshape(rows, ex.F), up.float().reshape(rows, ex.F)
        sg = torch.sigmoid(gf)
        silu = gf * sg
        d_up = d_act * silu
        d_gate = d_act * uf * (sg * (1 + gf * (1 - sg)))
        d_gu = torch.stack((d_gate.view(rows, -1, 64), d_up.view(rows, -1, 64)), 2).reshape(rows, 2 * ex.F)
        d_xp = grouped(ex.w_gu_t, d_gu.to(torch.bfloat16).contiguous(), ex.H, ex.H).float()
        dx = torch.zeros(T, ex.H, dtype=torch.float32, device=gout.device)
        dx.index_add_(0, tok, d_xp[slots])
        # router backward
        p = torch.softmax(logits, -1)
        chosen = idx.long().view(T, k)
        if ex.renorm:
            pc = p.gather(1, chosen)
            s = pc.sum(1, keepdim=True)
            d_pc = (dw - (dw * pc).sum(1, keepdim=True) / s) / s
        else:
            d_pc = dw
        dp = torch.zeros_like(p).scatter_add_(1, chosen, d_pc)
        dlog = p * (dp - (dp * p).sum(1, keepdim=True))
        dx += K.linear(dlog.to(torch.bfloat16).contiguous(), ex.router_t, out_dtype=torch.float32)
        return dx.to(gout.dtype), gout, None, None


def moe_ffn_autograd(x: torch.Tensor, h: torch.Tensor, experts: FrozenExperts, anchor: torch.Tensor) -> torch.Tensor:
    """h + MoE(x), differentiable in x and h (``anchor``: any tensor requiring grad)."""
    if not x.is_cuda:
        return _moe_reference_autograd(x, h, experts)
    return _MoEFFN.apply(x, h, anchor, experts)


def moe_ffn_lora(x: torch.Tensor, h: torch.Tensor, ex: FrozenExperts, gu_adapters, down_adapters, scale: float, *,
                 dropout: float = 0.0, training: bool = False) -> torch.Tensor:
    """h + MoE(x) with LoRA adapters on every expert's gate / up / down projection.

    ``gu_adapters[e]`` adapts expert e's interleaved gate / up rows (its B is
    block-masked so gate rows use the gate block of A and up rows the up block),
    ``down_adapters[e]`` its down projection; either list may hold None.  Routing
    is the top-k of the router softmax (renormalised when the model says so) with
    gradients through the routing weights; the experts run one after another on
    their routed rows through the differentiable LoRA linear (tcgen05 GEMMs on
    the GPU), as PEFT-adapted expert modules run in the reference's LLaDA-MoE
    (configs/gsm8k_llada_moe_3090.toml ``[vrpo_lora]`` targets gate/up/down_proj).
    """
    from .lora import lora_linear

    T, E, Fd, H, k = x.shape[0], ex.E, ex.F, ex.H, ex.k
    logits = x.float() @ ex.router.float().t()
    p = torch.softmax(logits, -1)
    order = torch.sort(-p.detach(), dim=-1, stable=True).indices[:, :k]
    w = p.gather(1, order)
    if ex.renorm:
        w = w / w.sum(1, keepdim=True)
    flat = order.reshape(-1)
    perm = torch.sort(flat, stable=True).indices
    counts = torch.bincount(flat, minlength=E).tolist()      # one host read per layer
    tok, slot = perm // k, perm % k
    out = h.float()
    xb = x.to(torch.bfloat16)
    start = 0
    for e, c in enumerate(counts):
        if c == 0:
            continue
        rows, slots = tok[start:start + c], slot[start:start + c]
        start += c
        gu = lora_linear(xb[rows], ex.w_gu[e * 2 * Fd:(e + 1) * 2 * Fd], gu_adapters[e], scale, dropout=dropout,
                         training=training)
        g, u = _swiglu_split(gu)
        act = (F.silu(g.float()) * u.float()).reshape(c, Fd).to(torch.bfloat16)
        ye = lora_linear(act, ex.w_down[e * H:(e + 1) * H], down_adapters[e], scale, dropout=dropout,
                         training=training)
        out = out.index_add(0, rows, ye.float() * w[rows, slots][:, None])
    return out.to(torch.bfloat16)


def _moe_reference_autograd(x, h, ex: FrozenExperts):
    """Plain PyTorch (CPU) version with autograd through routing weights."""
    p = torch.softmax(x.float() @ ex.router.float().t(), -1)
    order = torch.sort(-p.detach(), dim=-1, stable=True).indices[:, : ex.k]
    w = p.gather(1, order)
    if ex.renorm:
        w = w / w.sum(1, keepdim=True)
    out = h.float()
    E, H, Fd = ex.E, ex.H, ex.F
    for e in range(E):
        rows, slot = (order == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        gu = x[rows].float() @ ex.w_gu[e * 2 * Fd:(e + 1) * 2 * Fd].float().t()
        g, u = _swiglu_split(gu)
        act = (F.silu(g) * u).reshape(rows.numel(), Fd)
        yv = act @ ex.w_down[e * H:(e + 1) * H].float().t()
        out = out.index_add(0, rows, yv * w[rows, slot][:, None])
    return out.to(torch.bfloat16)
