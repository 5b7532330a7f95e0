"""Expert parallelism for the MoE layer: experts sharded over ranks, tokens exchanged.

Rank r owns experts [r * E / W, (r + 1) * E / W) and processes its own tokens
(data parallel outside the expert layer).  Per MoE layer:

* ``ExpertParallelMoE`` (the fused path): router GEMM + top-k on the local
  tokens, then ``ep_exchange`` phase 0 exchanges the per-expert counts through
  a symmetric table and stores every (token, choice) row straight into the
  owner's symmetric receive buffer over NVLink; the owner runs its local
  experts with the grouped tcgen05 GEMMs (tile list built on the device from
  the exchanged counts) into a symmetric output buffer; phase 1 pulls every
  token's k expert rows back from their owners and adds the weighted sum to the
  residual.  No host synchronisation, so the layer can be captured in a graph.
* ``NcclExpertParallelMoE`` (the baseline): the same routing, then
  ``all_to_all_single`` of counts and of sorted token rows (split sizes read on
  the host), local experts, and the reverse all-to-all.

Both give the single-GPU layer's result: the combine adds the expert rows in
choice order with fp32 accumulation.
"""

from __future__ import annotations

import torch

from ..ops import _ext, workspace
from ..ops import kernels as K


class _Routing:
    def __init__(self, max_tokens: int, E: int, k: int, device):
        rows = max_tokens * k
        i32 = dict(dtype=torch.int32, device=device)
        self.logits = torch.empty(max_tokens, E, dtype=torch.float32, device=device)
        self.idx = torch.empty(rows, **i32)
        self.w = torch.empty(rows, dtype=torch.float32, device=device)
        self.counts = torch.zeros(E, **i32)


class ExpertParallelMoE:
    """Fused expert-parallel MoE exchange over symmetric memory."""

    def __init__(self, group, *, experts: int, top_k: int, hidden: int, ffn: int, max_tokens: int, device,
                 blocks: int = 132, wait_limit_ns: int = 0):
        """``wait_limit_ns`` bounds every cross-rank wait of the exchange kernels (0: two seconds)."""
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if experts % self.world:
            raise ValueError(f"{experts} experts cannot be split over {self.world} ranks")
        if hidden % 128 or (2 * ffn) % 128:
            raise ValueError("hidden and 2 * ffn must be multiples of 128")
        self.E, self.k, self.H, self.F = experts, top_k, hidden, ffn
        self.E_local = experts // self.world
        self.max_tokens = max_tokens
        self.device = torch.device(device)
        self.blocks = blocks
        self.wait_limit_ns = int(wait_limit_ns)
        # worst case: every rank routes every choice of every token to this rank
        self.r_max = max_tokens * top_k * self.world
        self._table = symm.empty(self.world * experts, dtype=torch.int32, device=self.device)
        self._recv_x = symm.empty(self.r_max, hidden, dtype=torch.bfloat16, device=self.device)
        self._recv_y = symm.empty(self.r_max, hidden, dtype=torch.bfloat16, device=self.device)
        hs = [symm.rendezvous(t, group) for t in (self._table, self._recv_x, self._recv_y)]
        self._tables, self._xs, self._ys = (list(h.buffer_ptrs) for h in hs)
        self._pads = list(hs[0].signal_pad_ptrs)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.route = _Routing(max_tokens, experts, top_k, self.device)
        i32 = dict(dtype=torch.int32, device=self.device)
        self.cursor = torch.zeros(experts, **i32)
        self.slot_of = torch.empty(max_tokens * top_k, **i32)
        self.local_offsets = torch.zeros(self.E_local + 1, **i32)
        self.act = torch.empty(self.r_max, ffn, dtype=torch.bfloat16, device=self.device)
        tiles_m = max(2 * ffn, hidden) // 128
        cap = tiles_m * (-(-self.r_max // 32) + self.E_local)
        self.tiles = torch.zeros(2, cap * 4, **i32)
        self.total = torch.zeros(2, **i32)

    def moe_ffn(self, x, h, layer, config):
        """Hook of :class:`~online_speculation_b200.models.moe.MoEDiffusionModel` (one MoE layer)."""
        return self.ffn(x, h, layer.router, layer.w_gu, layer.w_down, renorm=config.norm_topk_prob)

    def ffn(self, x: torch.Tensor, h: torch.Tensor, router: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor,
            *, renorm: bool = False) -> torch.Tensor:
        """h += MoE(x) in place; ``w_gu`` [E_local * 2F, H] and ``w_down`` [E_local * H, F] are this rank's experts."""
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the expert-parallel buffers ({self.max_tokens})")
        if router.shape[0] != self.E or w_gu.shape[0] != self.E_local * 2 * self.F or \
                w_down.shape[0] != self.E_local * self.H:
            raise ValueError("router / local expert weights do not match the expert-parallel layout")
        ext = _ext.require()
        rt = self.route
        rows = T * self.k
        logits = K.linear(x, router, out=rt.logits[:T], out_dtype=torch.float32)
        rt.counts.zero_()
        ext.moe_route(logits, self.k, renorm, rt.idx[:rows], rt.w[:rows], rt.counts)
        st = workspace.status(self.device)
        args = (self._tables, self._xs, self._ys, self._pads, self.epoch, self.r_max, rt.counts, rt.idx, rt.w, x,
                self.cursor, self.slot_of, self.local_offsets, h, self.E, self.k, self.rank, self.blocks)
        ext.ep_exchange(*args, 0, st, self.wait_limit_ns)
        # local experts over the received rows (tile list built on the device from the exchanged counts)
        bn = K.moe_pick_bn(rows, self.E_local)
        ws, ctr = workspace.gemm_workspace(self.device), workspace.gemm_counters(self.device)
        tm_gu, tm_dn = 2 * self.F // 128, self.H // 128
        ext.grouped_tiles(self.local_offsets, self.E_local, tm_gu, bn, self.tiles[0], self.total[0:1])
        ext.grouped_gemm(w_gu, self._recv_x, self.act, 1, self.tiles[0], self.total[0:1], self.E_local, bn, ws, ctr,
                         st)
        ext.grouped_tiles(self.local_offsets, self.E_local, tm_dn, bn, self.tiles[1], self.total[1:2])
        ext.grouped_gemm(w_down, self.act, self._recv_y, 0, self.tiles[1], self.total[1:2], self.E_local, bn, ws,
                         ctr, st)
        ext.ep_exchange(*args, 1, st, self.wait_limit_ns)
        return h


class NcclExpertParallelMoE:
    """Baseline: all-to-all exchange through NCCL (split sizes synchronised to the host)."""

    def __init__(self, group, *, experts: int, top_k: int, hidden: int, ffn: int, max_tokens: int, device):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.E, self.k, self.H, self.F = experts, top_k, hidden, ffn
        self.E_local = experts // self.world
        self.device = torch.device(device)
        self.route = _Routing(max_tokens, experts, top_k, self.device)
        self.buffers = K.MoEBuffers(max_tokens * top_k * self.world, self.E_local, 1, hidden, ffn, self.device)

    def moe_ffn(self, x, h, layer, config):
        return self.ffn(x, h, layer.router, layer.w_gu, layer.w_down, renorm=config.norm_topk_prob)

    def ffn(self, x, h, router, w_gu, w_down, *, renorm: bool = False):
        import torch.distributed as dist

        T = x.shape[0]
        rows = T * self.k
        rt = self.route
        logits = K.linear(x, router, out=rt.logits[:T], out_dtype=torch.float32)
        rt.counts.zero_()
        _ext.require().moe_route(logits, self.k, renorm, rt.idx[:rows], rt.w[:rows], rt.counts)
        idx = rt.idx[:rows].long()
        owner = idx // self.E_local
        order = torch.sort(owner * self.E + idx, stable=True).indices     # by owner, then expert
        send = x[order // self.k]
        send_counts = torch.bincount(owner, minlength=self.world)
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        sc, rc = send_counts.tolist(), recv_counts.tolist()
        recv = torch.empty(sum(rc), self.H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(recv, send, rc, sc, group=self.group)
        send_e = (idx[order] % self.E_local).int()
        recv_e = torch.empty(sum(rc), dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_e, send_e, rc, sc, group=self.group)
        # local experts: a one-choice MoE over the received rows with the expert forced by recv_e
        y = _local_experts(recv, recv_e, w_gu, w_down, self.E_local, self.F, self.buffers)
        back = torch.empty(rows, self.H, dtype=x.dtype, device=x.device)
        dist.all_to_all_single(back, y, sc, rc, group=self.group)
        out = torch.empty_like(back)
        out[order] = back
        contrib = (out.view(T, self.k, self.H).float() * rt.w[:rows].view(T, self.k, 1)).sum(1)
        h.copy_((h.float() + contrib).to(h.dtype))
        return h


def _local_experts(xr: torch.Tensor, expert: torch.Tensor, w_gu, w_down, E_local: int, F: int, b: K.MoEBuffers):
    """Rows ``xr`` through their assigned local experts with the grouped GEMMs; returns [R, H]."""
    ext = _ext.require()
    R, H = xr.shape
    if R == 0:
        return torch.empty(0, H, dtype=xr.dtype, device=xr.device)
    counts = torch.bincount(expert.long(), minlength=E_local).int()
    b.counts[:E_local].copy_(counts)
    ext.moe_offsets(b.counts[:E_local], b.offsets[:E_local + 1], b.cursor[:E_local])
    slot = torch.empty(R, dtype=torch.int32, device=xr.device)
    ext.moe_dispatch(xr, expert.contiguous(), b.cursor[:E_local], b.xp, slot)
    bn = K.moe_pick_bn(R, E_local)
    ws, ctr, st = workspace.gemm_workspace(xr.device), workspace.gemm_counters(xr.device), workspace.status(xr.device)
    ext.grouped_tiles(b.offsets[:E_local + 1], E_local, 2 * F // 128, bn, b.tiles[0], b.total[0:1])
    ext.grouped_gemm(w_gu, b.xp[:R], b.act[:R], 1, b.tiles[0], b.total[0:1], E_local, bn, ws, ctr, st)
    ext.grouped_tiles(b.offsets[:E_local + 1], E_local, H // 128, bn, b.tiles[1], b.total[1:2])
    ext.grouped_gemm(w_down, b.act[:R], b.y[:R], 0, b.tiles[1], b.total[1:2], E_local, bn, ws, ctr, st)
    return b.y[:R][slot.long()]


__all__ = ["ExpertParallelMoE", "NcclExpertParallelMoE"]
