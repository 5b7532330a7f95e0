"""Batched forward pass of a decoder over a paged KV cache on the sm_100a kernels.

One :meth:`ModelRunner.forward` call processes a packed batch of sequences,
each contributing ``q_len`` new tokens (prefill chunks, single-token decode,
speculative verification blocks), and writes their K/V into the cache.  Per
layer it launches: RMSNorm -> QKV GEMM (+bias) -> Q/K-norm + RoPE + paged K/V
store -> paged attention -> O GEMM (+residual) -> RMSNorm -> gate/up GEMM with
fused SwiGLU -> down GEMM (+residual).  Under tensor parallelism the O and
down GEMMs produce partial sums that are reduced across ranks and added to the
residual stream by the following fused add+RMSNorm.

Replaces the reference's HF model forward inside
src/inference_scaling/arllm/backends/transformers_backend.py (decode loop
:869-1051) and DualViewDecoder.forward
(online-speculation/src/blockspec/parallel/backbone.py:243-291).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.decoder import DecoderWeights
from ..ops import kernels as K
from .kv_cache import KVCache


class Collectives:
    """Tensor-parallel reductions used by the runner.

    ``tp == 1``: identity.  Otherwise a communicator from
    :mod:`online_speculation_b200.parallel.symm` (fused peer-memory all-reduce
    + residual add + RMSNorm, or its NCCL baseline) provides
    ``partial_buffer`` / ``reduce_add_norm``.
    """

    def __init__(self, group=None, *, hidden: int = 0, max_tokens: int = 0, device=None, fused: bool = True,
                 push: bool | None = None, algorithm: str = "auto"):
        self.group = group
        self.impl = None
        if group is None:
            self.world, self.rank = 1, 0
            return
        import torch.distributed as dist

        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 1 and hidden:
            from ..parallel.symm import NcclCollectives, SymmetricCollectives

            if fused:
                self.impl = SymmetricCollectives(group, hidden, max_tokens, device, push=push, algorithm=algorithm)
            else:
                self.impl = NcclCollectives(group, hidden, max_tokens, device)

    def partial_buffer(self, T: int, scratch: torch.Tensor) -> torch.Tensor:
        return scratch if self.impl is None else self.impl.partial_buffer(T)

    def linear_into(self, x: torch.Tensor, w: torch.Tensor, part: torch.Tensor) -> torch.Tensor:
        """Row-parallel GEMM into a buffer from :meth:`partial_buffer` (the push
        communicator stores the tiles straight into every rank's receive slot)."""
        if self.impl is None:
            return K.linear(x, w, out=part, static_weights=True)
        return self.impl.linear_into(x, w, part)

    def reduce_add_norm(self, part, h, w, x, eps):
        if self.impl is not None:
            self.impl.reduce_add_norm(part, h, w, x, eps)
        else:
            self.all_reduce(part)
            K.rmsnorm(h, w, eps, out=x, residual=h, delta=part)

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(x, group=self.group)
        return x

    def gather_vocab(self, local: torch.Tensor, out: torch.Tensor, scratch: torch.Tensor) -> torch.Tensor:
        """[R, V_local] shards -> [R, world * V_local] full rows."""
        if self.world == 1:
            return local
        import torch.distributed as dist

        dist.all_gather_into_tensor(scratch, local.contiguous(), group=self.group)
        rows, width = local.shape
        out.view(rows, self.world, width).copy_(scratch.view(self.world, rows, width).transpose(0, 1))
        return out


@dataclass
class StepMeta:
    """Device metadata of one forward (all int32)."""

    ids: torch.Tensor         # [T]
    positions: torch.Tensor   # [T]
    slots: torch.Tensor       # [T]
    plan: K.AttentionPlan
    logit_rows: torch.Tensor | None  # [R] int64 row indices, None = all rows


class ModelRunner:
    def __init__(self, weights: DecoderWeights, cache: KVCache, *, collectives: Collectives | None = None,
                 max_tokens: int = 8192, max_logit_rows: int = 512):
        self.w = weights
        self.cfg = weights.config
        self.cache = cache
        self.comm = collectives or Collectives()
        self.device = weights.device
        self.max_tokens = max_tokens
        self.max_logit_rows = max_logit_rows
        self.q_slots = weights.heads.q_slots
        self.kv_slots = weights.heads.kv_slots
        self.vocab_local = weights.head.shape[0]
        self._buffers: dict[str, torch.Tensor] = {}
        # Buffers keep fixed storage for the runner's lifetime: CUDA graphs
        # captured over them must never see a reallocation.
        H, D, T, R = self.cfg.hidden_size, 128, max_tokens, max_logit_rows
        V = self.vocab_local * self.comm.world
        self._reserve = {
            "h": T * H, "x": T * H, "part": T * H, "sel": T * H, "dh": T * H, "dx": T * H, "xl": R * H, "xs": T * H,
            "qkv": T * (self.q_slots + 2 * self.kv_slots) * D, "q": T * self.q_slots * D,
            "att": T * self.q_slots * D, "act": T * weights.ffn_local,
            "logits_local": R * self.vocab_local, "logits_full": R * V, "logits_scratch": R * V,
            "draft_logits_keep": R * V,
        }

    # ---- buffers ----
    def _buf(self, name: str, shape, dtype=torch.bfloat16) -> torch.Tensor:
        numel = 1
        for s in shape:
            numel *= s
        b = self._buffers.get(name)
        if b is None:
            cap = max(numel, self._reserve.get(name, 0), 1)
            b = torch.empty(cap, dtype=dtype, device=self.device)
            self._buffers[name] = b
        elif b.numel() < numel or b.dtype != dtype:
            raise RuntimeError(f"runner buffer {name!r} needs {numel} elements but holds {b.numel()} "
                               f"(raise max_tokens / max_logit_rows)")
        return b[:numel].view(*shape)

    # ---- pieces ----
    def embed(self, ids: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        return K.embed(ids, self.w.embed, out)

    def attention_block(self, i: int, x: torch.Tensor, meta: StepMeta, *, wq=None, bias=None, q_norm=None,
                        k_norm=None, wo=None, residual: torch.Tensor | None = None) -> torch.Tensor:
        """x: normalised input [T, H].  Returns the attention output projected by O
        (added into ``residual`` in place when tp == 1, else a partial sum)."""
        lw = self.w.layers[i]
        T = x.shape[0]
        D = 128
        wq = lw.w_qkv if wq is None else wq
        bias = lw.b_qkv if bias is None and wq is lw.w_qkv else bias
        qkv = K.linear(x, wq, bias=bias, out=self._buf("qkv", (T, wq.shape[0])), static_weights=True)
        q = self._buf("q", (T, self.q_slots, D))
        kc, vc = self.cache.layer(i)
        K.rope_cache(qkv, meta.positions, meta.slots, self.w.inv_freq, q, kc, vc, self.q_slots, self.kv_slots,
                     q_norm=lw.q_norm if q_norm is None else q_norm, k_norm=lw.k_norm if k_norm is None else k_norm,
                     eps=self.cfg.rms_norm_eps)
        att = K.attention(q, kc, vc, meta.plan, out=self._buf("att", (T, self.q_slots, D)))
        wo = lw.w_o if wo is None else wo
        if self.comm.world == 1 and residual is not None:
            return K.linear(att.view(T, -1), wo, residual=residual, out=residual, static_weights=True)
        part = self.comm.partial_buffer(T, self._buf("part", (T, self.cfg.hidden_size)))
        return self.comm.linear_into(att.view(T, -1), wo, part)

    def mlp_block(self, i: int, x: torch.Tensor, residual: torch.Tensor | None) -> torch.Tensor:
        lw = self.w.layers[i]
        T = x.shape[0]
        act = K.linear(x, lw.w_gu, swiglu=True, out=self._buf("act", (T, lw.w_gu.shape[0] // 2)),
                       static_weights=True)
        if self.comm.world == 1 and residual is not None:
            return K.linear(act, lw.w_down, residual=residual, out=residual, static_weights=True)
        part = self.comm.partial_buffer(T, self._buf("part", (T, self.cfg.hidden_size)))
        return self.comm.linear_into(act, lw.w_down, part)

    def layer_stack(self, h: torch.Tensor, meta: StepMeta, layers: range) -> torch.Tensor:
        """Run decoder layers over the residual stream ``h`` (updated in place).

        Under tensor parallelism the buffer ``x`` holds, on return, the input of
        the layer after the range normalised by that layer's input norm (or by
        the final norm after the last layer).
        """
        eps = self.cfg.rms_norm_eps
        T = h.shape[0]
        x = self._buf("x", (T, self.cfg.hidden_size))
        L = self.cfg.num_hidden_layers
        tp = self.comm.world > 1
        for n, i in enumerate(layers):
            lw = self.w.layers[i]
            if n == 0 or not tp:
                K.rmsnorm(h, lw.in_norm, eps, out=x)
            part = self.attention_block(i, x, meta, residual=h)
            if tp:
                self.comm.reduce_add_norm(part, h, lw.post_norm, x, eps)
            else:
                K.rmsnorm(h, lw.post_norm, eps, out=x)
            part = self.mlp_block(i, x, residual=h)
            if tp:
                nxt = self.w.layers[i + 1].in_norm if i + 1 < L else self.w.final_norm
                self.comm.reduce_add_norm(part, h, nxt, x, eps)
        return h

    def logits(self, h: torch.Tensor, rows: torch.Tensor | None, *, normed: bool = False,
               out: torch.Tensor | None = None, gather: bool = True) -> torch.Tensor:
        """Final RMSNorm + vocabulary-parallel head on the selected rows -> fp32 [R, V]."""
        sel = h if rows is None else self._index_rows(h, rows)
        R = sel.shape[0]
        x = sel if normed else K.rmsnorm(sel, self.w.final_norm, self.cfg.rms_norm_eps,
                                         out=self._buf("xl", (R, self.cfg.hidden_size)))
        local = K.linear(x, self.w.head, out=self._buf("logits_local", (R, self.vocab_local), torch.float32),
                         out_dtype=torch.float32, static_weights=True)
        self.last_local_logits = local  # this rank's vocabulary shard (static buffer)
        if self.comm.world == 1 or not gather:
            return local
        full = out if out is not None else self._buf("logits_full", (R, self.vocab_local * self.comm.world),
                                                     torch.float32)
        scratch = self._buf("logits_scratch", (self.comm.world * R * self.vocab_local,), torch.float32)
        return self.comm.gather_vocab(local, full, scratch)

    def _index_rows(self, h: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
        out = self._buf("sel", (rows.numel(), h.shape[1]))
        torch.index_select(h, 0, rows, out=out)
        return out

    # ---- full forward ----
    def forward(self, meta: StepMeta, *, compute_logits: bool = True, gather: bool = True) -> torch.Tensor | None:
        """Decoder forward; returns fp32 logits of ``meta.logit_rows`` (all rows when None).

        Under tensor parallelism ``gather=False`` returns this rank's vocabulary
        shard (see :attr:`vocab_shard`) instead of full rows.
        """
        T = meta.ids.numel()
        h = self._buf("h", (T, self.cfg.hidden_size))
        self.embed(meta.ids, h)
        self.layer_stack(h, meta, range(self.cfg.num_hidden_layers))
        if not compute_logits:
            return None
        if self.comm.world > 1:
            # the last partial sum was folded and normalised already into x
            x = self._buf("x", (T, self.cfg.hidden_size))
            rows = meta.logit_rows
            sel = x if rows is None else self._index_rows(x, rows)
            return self.logits(sel, None, normed=True, gather=gather)
        return self.logits(h, meta.logit_rows)

    def forward_stats(self, meta: StepMeta, inv_temp: torch.Tensor | None, targets: torch.Tensor | None):
        """Decoder forward that scores ``meta.logit_rows`` without materialising logits.

        Returns fp32 (lse at T = 1, lse at T, log p and log q of ``targets``) per
        selected row from the fused head-statistics GEMM (one tensor-parallel rank only).
        """
        if self.comm.world > 1:
            raise ValueError("head statistics run on an unsharded vocabulary head")
        T = meta.ids.numel()
        h = self._buf("h", (T, self.cfg.hidden_size))
        self.embed(meta.ids, h)
        self.layer_stack(h, meta, range(self.cfg.num_hidden_layers))
        sel = h if meta.logit_rows is None else self._index_rows(h, meta.logit_rows)
        x = K.rmsnorm(sel, self.w.final_norm, self.cfg.rms_norm_eps,
                      out=self._buf("xs", (sel.shape[0], self.cfg.hidden_size)))
        return K.head_stats(x, self.w.head, inv_temp, targets)

    @property
    def vocab_shard(self) -> "K.VocabShard | None":
        """This rank's vocabulary slice for vocabulary-parallel sampling (None without TP)."""
        if self.comm.world == 1:
            return None
        if getattr(self, "_vocab_shard", None) is None:
            self._vocab_shard = K.VocabShard(self.comm.rank * self.vocab_local, self.vocab_local,
                                             self.vocab_local * self.comm.world, self.comm.group, self.comm.world)
        return self._vocab_shard


def build_meta(device, table: torch.Tensor, ids, positions, slots, q_lens, kv_lens, modes, group, logit_rows=None,
               tile_rows=None, kv_heads: int = 1) -> StepMeta:
    """Host-side helper: pack python lists into device metadata (eager paths and tests)."""
    def dev(v):
        return torch.as_tensor(v, dtype=torch.int32).to(device, non_blocking=True)

    plan = K.plan_attention(table, q_lens, kv_lens, modes, group, device, tile_rows=tile_rows, kv_heads=kv_heads)
    rows = None if logit_rows is None else torch.as_tensor(logit_rows, dtype=torch.int64).to(device)
    return StepMeta(dev(ids), dev(positions), dev(slots), plan, rows)
