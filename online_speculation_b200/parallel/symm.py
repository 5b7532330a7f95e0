"""Symmetric-memory tensor-parallel collectives for the decoder layers.

Buffers are allocated and exchanged with PyTorch's symmetric memory
(``torch.distributed._symmetric_memory``: cuMem allocations mapped into every
rank's address space over NVLink, plus zeroed signal pads).  The collective
itself is this package's sm_100a kernel pair (``csrc/comm.cu``): a two-shot
all-reduce over peer loads fused with the residual add and the next RMSNorm,
with bounded cross-rank barriers.  ``NcclCollectives`` is the NCCL baseline of
the same interface.
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

    def __init__(self, group, hidden: int, max_tokens: int, device, *, blocks: int = 132):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the fused all-reduce supports at most 8 ranks")
        self.device = torch.device(device)
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

    def partial_buffer(self, T: int) -> torch.Tensor:
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed the symmetric buffer ({self.max_tokens})")
        self._flip ^= 1
        return self._bufs[self._flip][:T]

    def reduce_add_norm(self, part: torch.Tensor, h: torch.Tensor, w: torch.Tensor, x: torch.Tensor, eps: float):
        flip = 0 if part.data_ptr() == self._bufs[0].data_ptr() else 1
        if part.data_ptr() != self._bufs[flip].data_ptr():
            raise ValueError("partials must live in this communicator's symmetric buffer")
        T = part.shape[0]
        _ext.require().allreduce_add_rmsnorm(self._parts_ptrs[flip], self._rows_ptrs, self._pads, self.epoch, h, w,
                                             x, T, self.rank, float(eps), self.blocks,
                                             workspace.status(self.device))
