"""Data-parallel gradient reduce-scatter and parameter all-gather over symmetric peer memory.

The sharded trainers (ZeRO-1: every rank owns a slice of the fp32 master weights and AdamW
moments) keep one flat fp32 gradient buffer and one flat bf16 parameter buffer per rank.
:class:`SymmetricDataParallel` allocates both as PyTorch symmetric memory (cuMem allocations
mapped into every rank's address space over NVLink) and moves data with this package's
kernels (``csrc/dp.cu``):

* :meth:`reduce_scatter` -- one launch per gradient bucket, issued on the trainer's side
  stream as soon as the bucket's gradients are complete, so it overlaps the rest of the
  backward pass: after a bounded cross-rank barrier, every rank sums its shard of the
  bucket over all ranks' buffers (peer loads, rank order -- the same sum on every rank)
  and scales it (the data-parallel mean);
* :meth:`all_gather` -- after the sharded AdamW, every rank stores its bf16 shard into
  every rank's parameter buffer (peer stores) between an opening and a closing barrier, so
  the next forward reads complete parameters.

``NcclDataParallel`` is the NCCL baseline of the same interface
(``reduce_scatter_tensor`` / ``all_gather_into_tensor``).
"""

from __future__ import annotations

import torch

from ..ops import _ext, workspace


class NcclDataParallel:
    """Baseline: NCCL reduce-scatter and all-gather on plain buffers."""

    symmetric = False

    def __init__(self, group, device):
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device)

    def allocate(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        return torch.zeros(numel, dtype=dtype, device=self.device)

    def reduce_scatter(self, grad: torch.Tensor, lo: int, hi: int, shard: torch.Tensor, scale: float) -> None:
        import torch.distributed as dist

        dist.reduce_scatter_tensor(shard, grad[lo:hi], group=self.group)
        if scale != 1.0:
            shard.mul_(scale)

    def all_gather(self, params: torch.Tensor, lo: int, hi: int, src: torch.Tensor) -> None:
        import torch.distributed as dist

        dist.all_gather_into_tensor(params[lo:hi], src, group=self.group)


class SymmetricDataParallel(NcclDataParallel):
    """Peer-memory reduce-scatter and all-gather kernels over symmetric buffers."""

    symmetric = True
    PAD_SLOTS = 3          # scatter, gather-start and gather-done flags (csrc/dp.h)

    def __init__(self, group, device, *, wait_limit_ns: int = 0):
        super().__init__(group, device)
        if not 2 <= self.world <= 8:
            raise ValueError("the peer-memory data-parallel collectives support 2 to 8 ranks")
        self.wait_limit_ns = int(wait_limit_ns)
        self.counters = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._ptrs: dict[int, list[int]] = {}      # buffer address -> every rank's address of it
        self._pads: list[int] | None = None
        self._keep = []

    def allocate(self, numel: int, dtype: torch.dtype) -> torch.Tensor:
        """A zeroed symmetric buffer (a collective call: every rank allocates in the same order)."""
        import torch.distributed._symmetric_memory as symm

        t = symm.empty(numel, dtype=dtype, device=self.device)
        t.zero_()
        h = symm.rendezvous(t, self.group)
        self._ptrs[t.data_ptr()] = [int(p) for p in h.buffer_ptrs]
        if self._pads is None:
            import torch.distributed as dist

            self._pads = [int(p) for p in h.signal_pad_ptrs]
            # the call counters start at zero: so must this rank's flags (a recycled allocation
            # may hold an earlier owner's), and every rank resets before any rank signals
            _ext.require().zero_device_bytes(self._pads[self.rank], self.PAD_SLOTS * 8 * 4)
            dist.barrier(group=self.group)
        self._keep.append((t, h))
        return t

    def _peers(self, buf: torch.Tensor) -> list[int]:
        base = buf.data_ptr()
        ptrs = self._ptrs.get(base)
        if ptrs is None:
            raise ValueError("the buffer was not allocated by this communicator")
        return ptrs

    def reduce_scatter(self, grad: torch.Tensor, lo: int, hi: int, shard: torch.Tensor, scale: float) -> None:
        n = (hi - lo) // self.world
        _ext.require().dp_reduce_scatter(self._peers(grad), self._pads, self.counters, self.rank, lo, n, shard,
                                         float(scale), workspace.status(self.device), self.wait_limit_ns)

    def all_gather(self, params: torch.Tensor, lo: int, hi: int, src: torch.Tensor) -> None:
        n = (hi - lo) // self.world
        _ext.require().dp_all_gather(self._peers(params), self._pads, self.counters, self.rank, src, lo, n,
                                     workspace.status(self.device), self.wait_limit_ns)


def make_data_parallel(group, device, kind: str = "symmetric", **kw):
    """``kind``: "symmetric" (peer-memory kernels) or "nccl"."""
    if kind == "symmetric":
        return SymmetricDataParallel(group, device, **kw)
    if kind == "nccl":
        return NcclDataParallel(group, device)
    raise ValueError(f"data-parallel collectives are 'symmetric' or 'nccl', not {kind!r}")
