"""Paged KV storage on the device plus the C++ page bookkeeping.

Storage is one tensor per K and V of shape [layers, pages, kv_heads, P, 128]
(P = 32 tokens per page), so one page of one head is a contiguous 8 KB block
that the attention kernel streams with 16-byte copies.  Page ownership,
reference counts, prefix sharing and copy-on-write forks live in the C++
``KVManager``.  Replaces the reference's per-request HF DynamicCache copies
(src/inference_scaling/arllm/backends/transformers_backend.py:368-416,
growing_cache.py) and blockspec's packed cache (online-speculation/src/blockspec/state.py).
"""

from __future__ import annotations

import torch

from ..ops import _ext
from ..ops import kernels as K

PAGE = K.PAGE_SIZE


class KVCache:
    def __init__(self, layers: int, kv_heads: int, num_pages: int, device, *, dtype=torch.bfloat16):
        ext = _ext.require()
        self.layers = layers
        self.kv_heads = kv_heads
        self.num_pages = num_pages
        self.device = torch.device(device)
        shape = (layers, num_pages, kv_heads, PAGE, 128)
        self.k = torch.zeros(shape, dtype=dtype, device=self.device)
        self.v = torch.zeros(shape, dtype=dtype, device=self.device)
        self.manager = ext.KVManager(num_pages, PAGE)
        self._pending_copies: list[int] = []

    @staticmethod
    def pages_for_budget(bytes_budget: int, layers: int, kv_heads: int) -> int:
        per_page = 2 * layers * kv_heads * PAGE * 128 * 2
        return max(1, int(bytes_budget // per_page))

    def layer(self, i: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.k[i], self.v[i]

    # ---- bookkeeping (host) ----
    def create(self) -> int:
        return self.manager.create()

    def release(self, seq: int) -> None:
        self.manager.release(seq)

    def length(self, seq: int) -> int:
        return self.manager.length(seq)

    def append(self, seq: int, n: int) -> list[int]:
        return self.manager.append(seq, n)

    def truncate(self, seq: int, n: int) -> None:
        self.manager.truncate(seq, n)

    def fork(self, seq: int, n: int) -> int:
        """Share the first n tokens of ``seq``; a partial boundary page is copied (queued)."""
        new, copies = self.manager.fork(seq, n)
        self._pending_copies.extend(copies)
        return new

    def flush_copies(self) -> None:
        """Run queued copy-on-write page copies on the current stream (all layers, K and V)."""
        if not self._pending_copies:
            return
        pairs = torch.tensor(self._pending_copies, dtype=torch.int32).view(-1, 3).to(self.device, non_blocking=True)
        K.page_copy(self.k, pairs)
        K.page_copy(self.v, pairs)
        self._pending_copies.clear()

    def fill_table(self, seqs: list[int], out: torch.Tensor) -> None:
        self.manager.fill_table(seqs, out)

    @property
    def free_pages(self) -> int:
        return self.manager.free_pages
