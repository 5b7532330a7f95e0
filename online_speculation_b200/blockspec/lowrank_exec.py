"""Fixed-capacity execution of noise-input drafting, replayed as CUDA graphs.

The executor owns one KV workspace per request, of shape ``[layers, 1, Hkv, capacity + scratch,
D]``. Every forward writes its own rows in place at their positions and attends over the whole
capacity. The visibility mask ``key <= position`` is computed on the device from the forward's
static position buffer. So a round copies only its token ids in and one scalar position offset.
The history is never moved, and a forward of a given ``(length, adapted)`` shape is one captured
graph. Rows beyond the committed length are stale but invisible. Warm-up and capture write only
into the ``scratch`` rows past the capacity.

The generation engine sees the history as a :class:`WorkspaceHistory` handle (its length), and
trims it by resetting that length; the workspace rows below the committed length never change
within a request. An online learner can therefore replay a draft against views of the workspace
(:meth:`GraphNoiseBranch.history`), and the adapters it updates in place are read by the graphs
at the next replay. Replacing parameter storage invalidates the graphs, and
:meth:`GraphNoiseBranch.validate` raises.

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/execution.py
(FixedShapeExecutor), decoding.py.
"""

from __future__ import annotations

import time
from dataclasses import dataclass

import torch
from torch import Tensor

from .diffusion import UniformNoise
from .generation import DraftBatch
from .lowrank import LowRankDecoder, NoiseBranch, NoiseDraft, WorkspaceLayer


@dataclass(frozen=True)
class WorkspaceHistory:
    length: int


class _Slot:
    """One fixed-shape forward: static ids / positions / adapter mask, logits out."""

    def __init__(self, branch: "GraphNoiseBranch", length: int, adapted: bool):
        dev = branch.k.device
        self.branch, self.length = branch, length
        self.ids = torch.zeros(1, length, dtype=torch.long, device=dev)
        self.base = torch.arange(length, device=dev)[None]
        self.positions = self.base + branch.capacity            # scratch rows until the first call
        self.mask = None
        if adapted:
            self.mask = torch.ones(1, length, dtype=torch.bool, device=dev)
            self.mask[:, 0] = False
        self.graph = None
        self.logits = None

    def run(self):
        b = self.branch
        allowed = (b.keys[None, :] <= self.positions[0][:, None])[None, None]
        layers = [WorkspaceLayer(b.k[i], b.v[i], self.positions[0]) for i in range(b.k.shape[0])]
        self.logits = b.model.forward_workspace(self.ids, self.positions, allowed, self.mask, layers)

    def capture(self):
        cur = torch.cuda.current_stream(self.ids.device)
        side = torch.cuda.Stream(device=self.ids.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            for _ in range(2):
                self.run()
        cur.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self.run()
        self.graph = graph

    def __call__(self, ids: Tensor, start: int) -> Tensor:
        self.ids.copy_(ids)
        torch.add(self.base, start, out=self.positions)
        if self.graph is None:
            self.run()
        else:
            self.graph.replay()
            self.branch.graph_replays += 1
        return self.logits.clone()


class GraphNoiseBranch(NoiseBranch):
    """:class:`NoiseBranch` over a fixed-capacity workspace; CUDA-graph replay on CUDA devices.

    Forwards longer than ``block_size`` (prefill) run eagerly through the same workspace path.
    Shapes not captured by :meth:`prepare` are captured on first use, and that time is counted
    in ``setup_seconds``."""

    def __init__(self, model: LowRankDecoder, noise: UniformNoise = UniformNoise(), block_size: int = 8, *,
                 capacity: int = 4096, use_cuda_graph: bool | None = None):
        super().__init__(model, noise, block_size)
        c = model.config
        p = model.lm_head.weight
        if capacity < 1:
            raise ValueError("capacity must be positive")
        self.capacity = capacity
        shape = (c.num_hidden_layers, 1, c.num_key_value_heads, capacity + block_size, c.head_dim)
        self.k = torch.zeros(shape, dtype=p.dtype, device=p.device)
        self.v = torch.zeros(shape, dtype=p.dtype, device=p.device)
        self.keys = torch.arange(capacity + block_size, device=p.device)
        self.use_cuda_graph = p.device.type == "cuda" if use_cuda_graph is None else use_cuda_graph
        if self.use_cuda_graph and p.device.type != "cuda":
            raise ValueError("CUDA graphs need a CUDA model")
        self.slots: dict = {}
        self.graph_replays = self.eager_forwards = 0
        self.setup_seconds = 0.0
        self._storage = self._signature()

    def _signature(self):
        return [(n, p.data_ptr(), p.dtype) for n, p in self.model.named_parameters()]

    def validate(self):
        if self._signature() != self._storage:
            raise RuntimeError("model parameter storage changed; build a new executor")

    @torch.no_grad()
    def prepare(self, lengths=None):
        """Capture the AR / verify (unadapted) and draft (adapted) shapes up to ``block_size``."""
        lengths = range(1, self.default_block_size + 1) if lengths is None else lengths
        for t in lengths:
            self._slot(t, False)
            if t >= 2:
                self._slot(t, True)

    def _slot(self, length: int, adapted: bool) -> _Slot:
        key = (length, adapted)
        if key not in self.slots:
            t0 = time.perf_counter()
            slot = _Slot(self, length, adapted)
            if self.use_cuda_graph:
                slot.capture()
                torch.cuda.synchronize(self.k.device)
            self.slots[key] = slot
            self.setup_seconds += time.perf_counter() - t0
        return self.slots[key]

    def cache_length(self, cache) -> int:
        return 0 if cache is None else cache.length

    def trim(self, cache: WorkspaceHistory, n: int) -> WorkspaceHistory:
        if not 0 <= n <= cache.length:
            raise ValueError("cannot extend a history by trimming")
        return WorkspaceHistory(n)

    def history(self, n: int):
        """Per-layer views of the first ``n`` workspace rows, valid until the request ends."""
        if n == 0:
            return None
        return tuple((self.k[i][:, :, :n], self.v[i][:, :, :n]) for i in range(self.k.shape[0]))

    def _forward(self, ids: Tensor, start: int, adapted: bool) -> Tensor:
        T = ids.shape[1]
        if start + T > self.capacity:
            raise ValueError(f"the request exceeds the workspace capacity of {self.capacity} positions")
        if T <= self.default_block_size:
            return self._slot(T, adapted)(ids, start)
        self.eager_forwards += 1
        slot = _Slot(self, T, adapted)
        return slot(ids, start)

    def ar(self, tokens: Tensor, cache=None, logits_to_keep: int = 0):
        start = self.cache_length(cache)
        if start == 0:
            self.validate()
        logits = self._forward(tokens, start, False)
        return ((logits[:, -logits_to_keep:] if logits_to_keep else logits),
                WorkspaceHistory(start + tokens.shape[1]))

    def draft(self, anchor: Tensor, cache, block_size: int, sampler, generator=None, feedback=None):
        start = self.cache_length(cache)
        noisy = self.noise.sample((1, block_size - 1), self.model.config.vocab_size, device=anchor.device,
                                  generator=generator)
        inputs = torch.cat((anchor, noisy), 1)
        logits = self._forward(inputs, start, True)
        root = sampler.sample_ar(logits[0, 0], generator)
        cand, q = sampler.propose(logits[0, 1:], generator)
        collect = feedback is not None and getattr(feedback, "learner", None) is not None
        route = None
        if collect:
            route = torch.ones_like(inputs, dtype=torch.bool)
            route[:, 0] = False
        return DraftBatch(torch.cat((anchor.new_tensor([[root]]), cand[None]), 1), cand, q,
                          WorkspaceHistory(start + 1), [root], inputs,
                          NoiseDraft(self.history(start), inputs, route) if collect else None, collect)


__all__ = ["GraphNoiseBranch", "WorkspaceHistory"]
