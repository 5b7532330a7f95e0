"""Dual-view drafting and verification on the sm_100a engine (batch one).

``KernelBranch`` serves a :class:`~online_speculation_b200.blockspec.model.DualViewDecoder`
with the package's kernels: its weights are converted once into the fused
kernel layouts (AR view) plus per-layer draft-attention tensors, the history
lives in paged KV, the AR view is the runner's ordinary forward and the draft
view is the same layer stack with each layer's draft projections and a
bidirectional block plan.  The draft pass writes its block K/V into the block's
slots, which the verify pass then overwrites, so the persistent history always
belongs to the AR view (online-speculation/src/blockspec/parallel/branches.py,
backbone.py:243-291).  Drop-in for ``MaskedAttentionBranch`` in ``generate``.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..engine.kv_cache import KVCache
from ..engine.runner import ModelRunner, build_meta
from ..models.decoder import DecoderConfig, build_weights
from ..ops import kernels as K
from .generation import DraftBatch
from .model import DualViewDecoder


@dataclass
class PagedHistory:
    seq: int
    length: int


def _decoder_config(c) -> DecoderConfig:
    return DecoderConfig(vocab_size=c.vocab_size, hidden_size=c.hidden_size, intermediate_size=c.intermediate_size,
                         num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads,
                         num_key_value_heads=c.num_key_value_heads, head_dim=c.head_dim, rope_theta=c.rope_theta,
                         rms_norm_eps=c.rms_norm_eps, attention_bias=c.attention_bias, qk_norm=True,
                         tie_word_embeddings=c.tie_word_embeddings, name="dual-view")


def _hf_state(model: DualViewDecoder, view: str) -> dict:
    """HF-named state dict of one view (for the kernel weight builder)."""
    c = model.config
    sd = {"model.embed_tokens.weight": model.embedding.weight, "model.norm.weight": model.norm.weight}
    if not c.tie_word_embeddings:
        sd["lm_head.weight"] = model.head.weight
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        a = getattr(layer.attention, view)
        for n in ("q", "k", "v", "o"):
            sd[p + f"self_attn.{n}_proj.weight"] = getattr(a, n).weight
            if c.attention_bias:
                sd[p + f"self_attn.{n}_proj.bias"] = getattr(a, n).bias
        sd[p + "self_attn.q_norm.weight"] = a.q_norm.weight
        sd[p + "self_attn.k_norm.weight"] = a.k_norm.weight
        sd[p + "mlp.gate_proj.weight"] = layer.gate.weight
        sd[p + "mlp.up_proj.weight"] = layer.up.weight
        sd[p + "mlp.down_proj.weight"] = layer.down.weight
        sd[p + "input_layernorm.weight"] = layer.input_norm.weight
        sd[p + "post_attention_layernorm.weight"] = layer.post_norm.weight
    return {k: v.detach() for k, v in sd.items()}


class KernelBranch:
    initial_ar_token = True
    input_budget_extra = 1

    def __init__(self, model: DualViewDecoder, *, device="cuda", kv_bytes: int = 1 << 30, max_tokens: int = 4096):
        c = model.config
        if c.head_dim != 128:
            raise ValueError("the sm_100a attention kernels need head_dim 128")
        self.config = c
        self.default_block_size = c.block_size
        cfg = _decoder_config(c)
        dev = torch.device(device)
        w = build_weights(cfg, _hf_state(model, "ar"), device=dev)
        dw = build_weights(cfg, _hf_state(model, "draft"), device=dev)
        self.draft_layers = [(lw.w_qkv, lw.b_qkv, lw.q_norm, lw.k_norm, lw.w_o) for lw in dw.layers]
        pages = KVCache.pages_for_budget(kv_bytes, cfg.num_hidden_layers, w.heads.kv_slots)
        self.runner = ModelRunner(w, KVCache(cfg.num_hidden_layers, w.heads.kv_slots, pages, dev),
                                  max_tokens=max_tokens)
        self.max_pages = -(-max_tokens // 32) + 1
        self.device = dev

    # -- cache protocol used by generate() --
    def cache_length(self, cache: PagedHistory | None) -> int:
        return 0 if cache is None else cache.length

    def trim(self, cache: PagedHistory, n: int) -> PagedHistory:
        self.runner.cache.truncate(cache.seq, n)
        cache.length = n
        return cache

    def release(self, cache: PagedHistory | None) -> None:
        if cache is not None:
            self.runner.cache.release(cache.seq)

    def _meta(self, cache: PagedHistory, tokens: list[int], mode: int, rows=None):
        r = self.runner
        n = len(tokens)
        slots = r.cache.append(cache.seq, n)
        table = torch.zeros(1, self.max_pages, dtype=torch.int32)
        r.cache.fill_table([cache.seq], table)
        G = r.q_slots // r.kv_slots
        return build_meta(self.device, table, tokens, list(range(cache.length, cache.length + n)), slots, [n],
                          [cache.length + n], [mode], G, logit_rows=rows, kv_heads=r.kv_slots)

    def ar(self, tokens: torch.Tensor, cache: PagedHistory | None = None, logits_to_keep: int = 0):
        if cache is None:
            cache = PagedHistory(self.runner.cache.create(), 0)
        ids = tokens[0].tolist()
        rows = list(range(len(ids) - logits_to_keep, len(ids))) if logits_to_keep else None
        meta = self._meta(cache, ids, 0, rows)
        logits = self.runner.forward(meta)
        cache.length += len(ids)
        return logits.float()[None], cache

    def draft(self, anchor: torch.Tensor, cache: PagedHistory, block_size: int, sampler, generator=None,
              feedback=None) -> DraftBatch:
        r = self.runner
        ids = [int(anchor[0, 0])] + [self.config.mask_token_id] * (block_size - 1)
        meta = self._meta(cache, ids, 1, list(range(block_size - 1)))
        h = r._buf("dh", (block_size, self.config.hidden_size))
        r.embed(meta.ids, h)
        x = r._buf("dx", (block_size, self.config.hidden_size))
        eps = self.config.rms_norm_eps
        for i, (wq, b, qn, kn, wo) in enumerate(self.draft_layers):
            lw = r.w.layers[i]
            K.rmsnorm(h, lw.in_norm, eps, out=x)
            r.attention_block(i, x, meta, wq=wq, bias=b, q_norm=qn, k_norm=kn, wo=wo, residual=h)
            K.rmsnorm(h, lw.post_norm, eps, out=x)
            r.mlp_block(i, x, residual=h)
        logits = r.logits(h, meta.logit_rows).float()
        # the block's draft K/V sit in the slots the verify pass will overwrite
        r.cache.truncate(cache.seq, cache.length)
        cand, q = sampler.propose(logits, generator)
        inputs = torch.tensor([ids], device=anchor.device)
        return DraftBatch(torch.cat((anchor, cand[None].to(anchor.device)), 1), cand, q, cache, [], inputs, None, False)
