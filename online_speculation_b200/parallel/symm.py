"""Symmetric-memory tensor-parallel collectives for the decoder layers.

Buffers are allocated and exchanged with PyTorch's symmetric memory
(``torch.distributed._symmetric_memory``: cuMem allocations mapped into every
rank's address space over NVLink, plus zeroed signal pads).  The collective
itself is this package's sm_100a kernels (``csrc/comm.cu``): a one-shot (up to
four ranks) or single-kernel two-shot all-reduce over peer loads fused with the
residual add and the next RMSNorm, with bounded cross-rank barriers.

Push mode (up to four ranks, opt-in): the row-parallel GEMM itself stores each
output tile into every rank's receive slot for this rank (``csrc/gemm.cu`` push
epilogue, peer stores over NVLink while the remaining tiles compute) and its
last CTA releases a completion flag on every rank; the reduction kernel then
waits for the flags and sums local memory only.

``NcclCollectives`` is the NCCL baseline of the same interface.
"""

from __future__ import annotations

import torch

from ..ops import _ext, workspace
from ..ops import kernels as K


class NcclCollectives:
    """Baseline: NCCL all-reduce then the fused add + RMSNorm kernel."""

    def __init__(self, group, hidden: int, max_tokens: int, device):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self._parts = torch.empty(2, max_tokens, hidden, dtype=torch.bfloat16, device=device)
        self._flip = 0

    def partial_buffer(self, T: int) -> torch.Tensor:
        self._flip ^= 1
        return self._parts[self._flip, :T]

    def linear_into(self, x: torch.Tensor, w: torch.Tensor, part: torch.Tensor) -> torch.Tensor:
        """Row-parallel GEMM ``part = x @ w.T`` into a buffer from :meth:`partial_buffer`."""
        return K.linear(x, w, out=part, static_weights=True)

    def reduce_add_norm(self, part: torch.Tensor, h: torch.Tensor, w: torch.Tensor, x: torch.Tensor, eps: float):
        import torch.distributed as dist

        dist.all_reduce(part, group=self.group)
        K.rmsnorm(h, w, eps, out=x, residual=h, delta=part)

    def all_reduce(self, t: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist

        dist.all_reduce(t, group=self.group)
        return t


class SymmetricCollectives(NcclCollectives):
    """Fused peer-memory all-reduce + residual + RMSNorm over NVLink."""

    PUSH_SLOT = 4          # flag slot of the pushing GEMMs (csrc/comm.h kPushSlot)
    MAX_RANKS = 8

    ALGORITHMS = {"auto": 0, "oneshot": 1, "twoshot": 2}

    def __init__(self, group, hidden: int, max_tokens: int, device, *, blocks: int = 132, push: bool | None = None,
                 algorithm: str = "auto", wait_limit_ns: int = 0):
        """``algorithm``: "auto" (one-shot up to four ranks, and above while each rank reads at most
        16 MiB of peer partials; two-shot otherwise), "oneshot" or "twoshot".
        ``wait_limit_ns``: limit of every cross-rank wait inside the kernels (0: two seconds); a wait
        that runs out records an error in the status word instead of hanging."""
        import os

        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-reduce supports at most 8 ranks")
        self.device = torch.device(device)
        if algorithm not in self.ALGORITHMS:
            raise ValueError(f"algorithm must be one of {sorted(self.ALGORITHMS)}")
        self.algorithm = self.ALGORITHMS[algorithm]
        self.wait_limit_ns = int(wait_limit_ns)
        self.blocks = blocks
        self.hidden = hidden
        self.max_tokens = max_tokens
        self._bufs = []
        self._handles = []
        for _ in range(2):
            t = symm.empty(max_tokens, hidden, dtype=torch.bfloat16, device=self.device)
            self._bufs.append(t)
            self._handles.append(symm.rendezvous(t, group))
        self._rows = symm.empty(max_tokens, hidden, dtype=torch.bfloat16, device=self.device)
        self._rows_h = symm.rendezvous(self._rows, group)
        self.epoch = torch.zeros(4, dtype=torch.int32, device=self.device)   # call counter, two arrival counters
        self._flip = 0
        self._parts_ptrs = [list(h.buffer_ptrs) for h in self._handles]
        self._rows_ptrs = list(self._rows_h.buffer_ptrs)
        self._pads = list(self._rows_h.signal_pad_ptrs)
        # Off unless asked for: measured on two B200s (7B verify round, bench.py --gpus 2) the
        # push variant ran 8147 tok/s against 8626 for the pull all-reduce -- the GEMM
        # epilogue's extra peer stores and its closing system fence cost more than the
        # overlap gains.
        self.push = bool(push) and self.world <= 4
        if self.push:
            # receive buffers [world, max_tokens, hidden] per flip; slot q holds rank q's partial
            self._recv = []
            self._recv_h = []
            for _ in range(2):
                t = symm.empty(self.world * max_tokens, hidden, dtype=torch.bfloat16, device=self.device)
                self._recv.append(t)
                self._recv_h.append(symm.rendezvous(t, group))
            slot_bytes = max_tokens * hidden * 2
            self._push_dsts = [[int(p) + self.rank * slot_bytes for p in h.buffer_ptrs] for h in self._recv_h]
            self._push_local = [[int(h.buffer_ptrs[self.rank]) + q * slot_bytes for q in range(self.world)]
                                for h in self._recv_h]
            self._push_flags = [int(p) + (self.PUSH_SLOT * self.MAX_RANKS + self.rank) * 4 for p in self._pads]
            self._push_count = torch.zeros(1, dtype=torch.int32, device=self.device)

    def partial_buffer(self, T: int) -> torch.Tensor:
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the symmetric buffer ({self.max_tokens})")
        self._flip ^= 1
        if self.push:
            start = self.rank * self.max_tokens
            return self._recv[self._flip][start:start + T]
        return self._bufs[self._flip][:T]

    def _push_flip(self, part: torch.Tensor) -> int | None:
        if not self.push:
            return None
        for f in (0, 1):
            if part.data_ptr() == self._recv[f].data_ptr() + self.rank * self.max_tokens * self.hidden * 2:
                return f
        return None

    def linear_into(self, x: torch.Tensor, w: torch.Tensor, part: torch.Tensor) -> torch.Tensor:
        f = self._push_flip(part)
        if f is None:
            return K.linear(x, w, out=part, static_weights=True)
        _ext.require().gemm_push(w, x, part, self._push_dsts[f], self._push_flags, self.epoch, self._push_count,
                                 True, workspace.gemm_workspace(x.device), workspace.gemm_counters(x.device),
                                 workspace.status(x.device), True)
        return part

    def reduce_add_norm(self, part: torch.Tensor, h: torch.Tensor, w: torch.Tensor, x: torch.Tensor, eps: float):
        pf = self._push_flip(part)
        if pf is not None:
            T = part.shape[0]
            _ext.require().allreduce_pushed_add_rmsnorm(self._push_local[pf], self._pads, self.epoch, h, w, x, T,
                                                        self.rank, float(eps), self.blocks,
                                                        workspace.status(self.device), self.wait_limit_ns)
            return
        flip = 0 if part.data_ptr() == self._bufs[0].data_ptr() else 1
        if part.data_ptr() != self._bufs[flip].data_ptr():
            raise ValueError("partials must live in this communicator's symmetric buffer")
        T = part.shape[0]
        _ext.require().allreduce_add_rmsnorm(self._parts_ptrs[flip], self._rows_ptrs, self._pads, self.epoch, h, w,
                                             x, T, self.rank, float(eps), self.blocks,
                                             workspace.status(self.device), self.algorithm, self.wait_limit_ns)
