"""Dual-view decoder: one Qwen3-shaped backbone with two attention projection sets.

The ``ar`` view is the ordinary causal decoder and owns the persistent KV
history.  The ``draft`` view re-reads that history read-only and attends
bidirectionally inside a block ``[anchor, MASK, ..., MASK]``; everything but
the attention projections (embeddings, norms, MLPs, head) is shared.
Semantics follow online-speculation/src/blockspec/parallel/backbone.py:15-321.

This PyTorch module is the training / oracle path (distillation, online
suffix replay with ``forward_suffix``, audits).  Serving on B200 uses the same
weights on the sm_100a kernels through :mod:`online_speculation_b200.blockspec.kernel_branch`.

Parameter names match the reference's own state-dict keys
(``layers.{i}.attention.{ar,draft}.{q,k,v,o,q_norm,k_norm}``, ``input_norm``,
``post_norm``, ``gate``, ``up``, ``down``, ``embedding``, ``norm``, ``head``) so
``blockspec-dual-view-v1`` checkpoints are interchangeable.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass

import torch
import torch.nn.functional as F
from torch import Tensor, nn

Cache = tuple  # tuple[(k [B, Hkv, T, D], v [B, Hkv, T, D]), ...] per layer


def cache_length(cache) -> int:
    if cache is not None and not cache:
        raise ValueError("empty cache tuple; use None for an empty prefix")
    return 0 if cache is None else cache[0][0].shape[2]


def trim_cache(cache, length: int):
    """Keep the first ``length`` positions of every layer (detached)."""
    if length < 0 or length > cache_length(cache):
        raise ValueError("cannot extend a cache by trimming")
    if cache is None or length == 0:
        return None
    return tuple((k[:, :, :length].detach(), v[:, :, :length].detach()) for k, v in cache)


@dataclass(frozen=True)
class DualViewConfig:
    vocab_size: int = 32
    hidden_size: int = 64
    intermediate_size: int = 128
    num_hidden_layers: int = 2
    num_attention_heads: int = 4
    num_key_value_heads: int = 2
    head_dim: int = 16
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0
    attention_bias: bool = False
    tie_word_embeddings: bool = True
    block_size: int = 4
    mask_token_id: int = 1
    eos_token_id: int | None = None

    def __post_init__(self):
        dims = (self.vocab_size, self.hidden_size, self.intermediate_size, self.num_hidden_layers,
                self.num_attention_heads, self.num_key_value_heads, self.head_dim)
        if min(dims) < 1:
            raise ValueError("positive model dimensions required")
        if self.head_dim % 2 or self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("even head width and integral query/KV ratio required")
        if self.block_size < 2 or not 0 <= self.mask_token_id < self.vocab_size:
            raise ValueError("invalid mask token or block size")
        if self.eos_token_id is not None and not 0 <= self.eos_token_id < self.vocab_size:
            raise ValueError("invalid EOS token")
        if not (math.isfinite(self.rms_norm_eps) and self.rms_norm_eps > 0):
            raise ValueError("positive finite normalization epsilon required")
        if not (math.isfinite(self.rope_theta) and self.rope_theta > 1):
            raise ValueError("finite rotary base greater than one required")

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_public(cls, data: dict) -> "DualViewConfig":
        """From a HF ``config.json`` of a Qwen3 (or dual-view) checkpoint."""
        if data.get("model_type") not in ("qwen3", "orthrus"):
            raise ValueError("the dual-view importer requires a Qwen3 checkpoint")
        if data.get("hidden_act", "silu") != "silu":
            raise ValueError("SwiGLU activation required")
        if data.get("use_sliding_window", False) or any(t != "full_attention" for t in data.get("layer_types", [])):
            raise ValueError("this backbone implements full attention")
        rope = data.get("rope_parameters") or data.get("rope_scaling") or {}
        if rope.get("rope_type", rope.get("type", "default")) != "default":
            raise ValueError("ordinary RoPE required")
        names = cls.__dataclass_fields__
        values = {k: data[k] for k in names if k in data}
        if "rope_theta" in rope:
            values["rope_theta"] = rope["rope_theta"]
        required = set(names) - {"attention_bias", "tie_word_embeddings", "eos_token_id"}
        missing = required - values.keys()
        if missing:
            raise ValueError(f"missing architecture fields: {sorted(missing)}")
        return cls(**values)


class RMSNorm(nn.Module):
    def __init__(self, width: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.epsilon = eps

    def forward(self, x: Tensor) -> Tensor:
        work = x.float()
        normed = work * torch.rsqrt(work.square().mean(-1, keepdim=True) + self.epsilon)
        return normed.to(x.dtype) * self.weight


class AttentionView(nn.Module):
    """One projection set with per-head Q/K RMSNorm."""

    def __init__(self, c: DualViewConfig):
        super().__init__()
        qw, kvw = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
        self.q = nn.Linear(c.hidden_size, qw, bias=c.attention_bias)
        self.k = nn.Linear(c.hidden_size, kvw, bias=c.attention_bias)
        self.v = nn.Linear(c.hidden_size, kvw, bias=c.attention_bias)
        self.o = nn.Linear(qw, c.hidden_size, bias=c.attention_bias)
        self.q_norm = RMSNorm(c.head_dim, c.rms_norm_eps)
        self.k_norm = RMSNorm(c.head_dim, c.rms_norm_eps)


def rotate(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    half = x.shape[-1] // 2
    a, b = x[..., :half], x[..., half:]
    return torch.cat((a * cos[..., :half] - b * sin[..., :half], b * cos[..., half:] + a * sin[..., half:]), -1)


class DualAttention(nn.Module):
    def __init__(self, c: DualViewConfig):
        super().__init__()
        self.config = c
        self.ar = AttentionView(c)
        self.draft = AttentionView(c)

    def forward(self, x, view, cache, rotary, allowed):
        c = self.config
        B, T, _ = x.shape
        p = getattr(self, view)
        q = p.q_norm(p.q(x).view(B, T, -1, c.head_dim)).transpose(1, 2)
        k = p.k_norm(p.k(x).view(B, T, -1, c.head_dim)).transpose(1, 2)
        v = p.v(x).view(B, T, -1, c.head_dim).transpose(1, 2)
        cos, sin = rotary
        q, k = rotate(q, cos, sin), rotate(k, cos, sin)
        if cache is not None:
            k, v = torch.cat((cache[0], k), 2), torch.cat((cache[1], v), 2)
        g = c.num_attention_heads // c.num_key_value_heads
        kk, vv = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
        scores = (q.float() @ kk.float().transpose(-1, -2)) * c.head_dim ** -0.5
        if allowed is not None:
            scores = scores.masked_fill(~allowed, float("-inf"))
        out = (scores.softmax(-1).to(q.dtype) @ vv).transpose(1, 2).reshape(B, T, -1)
        return p.o(out), (k, v)


class DualLayer(nn.Module):
    def __init__(self, c: DualViewConfig):
        super().__init__()
        self.attention = DualAttention(c)
        self.input_norm = RMSNorm(c.hidden_size, c.rms_norm_eps)
        self.post_norm = RMSNorm(c.hidden_size, c.rms_norm_eps)
        self.gate = nn.Linear(c.hidden_size, c.intermediate_size, bias=False)
        self.up = nn.Linear(c.hidden_size, c.intermediate_size, bias=False)
        self.down = nn.Linear(c.intermediate_size, c.hidden_size, bias=False)

    def forward(self, x, view, cache, rotary, allowed):
        a, kv = self.attention(self.input_norm(x), view, cache, rotary, allowed)
        x = x + a
        n = self.post_norm(x)
        return x + self.down(F.silu(self.gate(n)) * self.up(n)), kv


@dataclass
class DraftBoundary:
    """Input of the first replayed layer, frozen for online suffix replay."""

    hidden: Tensor
    rotary: tuple
    allowed: Tensor | None
    start_layer: int
    history_length: int

    def detached(self) -> "DraftBoundary":
        return DraftBoundary(self.hidden.detach().clone(), tuple(t.detach().clone() for t in self.rotary),
                             None if self.allowed is None else self.allowed.detach().clone(), self.start_layer,
                             self.history_length)


@dataclass
class BackboneOutput:
    hidden: Tensor
    cache: Cache | None
    logits: Tensor | None
    boundary: DraftBoundary | None = None


class DualViewDecoder(nn.Module):
    def __init__(self, config: DualViewConfig = DualViewConfig()):
        super().__init__()
        self.config = config
        self.embedding = nn.Embedding(config.vocab_size, config.hidden_size)
        self.layers = nn.ModuleList(DualLayer(config) for _ in range(config.num_hidden_layers))
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.register_buffer("frequencies", self._frequencies(self.embedding.weight.device), persistent=False)
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, std=0.02)
                if isinstance(m, nn.Linear) and m.bias is not None:
                    nn.init.zeros_(m.bias)
        self.tie_weights()
        self.initialize_draft_from_ar()
        self.source: dict = {}

    def tie_weights(self):
        if self.config.tie_word_embeddings:
            self.head.weight = self.embedding.weight

    def _frequencies(self, device):
        # the fp32 table is formed on the host, then moved
        idx = torch.arange(0, self.config.head_dim, 2, dtype=torch.float32)
        return (1.0 / (self.config.rope_theta ** (idx / self.config.head_dim))).to(device)

    def _apply(self, fn, recurse=True):
        super()._apply(fn, recurse=recurse)
        self.frequencies = self._frequencies(self.embedding.weight.device)
        return self

    @torch.no_grad()
    def initialize_draft_from_ar(self):
        for layer in self.layers:
            layer.attention.draft.load_state_dict(layer.attention.ar.state_dict())

    def train_draft_only(self):
        self.requires_grad_(False)
        for layer in self.layers:
            layer.attention.draft.requires_grad_(True)
        return self.train()

    def _rotary(self, positions: Tensor, dtype):
        phase = positions.float()[..., None] * self.frequencies
        phase = torch.cat((phase, phase), -1)[:, None]
        return phase.cos().to(dtype), phase.sin().to(dtype)

    def forward(self, tokens: Tensor, *, view: str = "ar", cache=None, positions=None, allowed=None,
                logits_to_keep: int = 0, compute_logits: bool = True, capture_layer: int | None = None
                ) -> BackboneOutput:
        if view not in ("ar", "draft"):
            raise ValueError("view must be ar or draft")
        if tokens.ndim != 2 or tokens.shape[1] < 1:
            raise ValueError("nonempty tokens[batch, time] required")
        if capture_layer is not None and (view != "draft" or not 0 <= capture_layer < len(self.layers)):
            raise ValueError("draft capture requires a valid layer boundary")
        B, T = tokens.shape
        past = cache_length(cache)
        if positions is None:
            positions = torch.arange(past, past + T, device=tokens.device)[None]
        if allowed is None and view == "ar":
            q = torch.arange(past, past + T, device=tokens.device)
            allowed = (torch.arange(past + T, device=tokens.device)[None] <= q[:, None])[None, None]
        h = self.embedding(tokens)
        rotary = self._rotary(positions, h.dtype)
        new_cache, boundary = [], None
        for i, layer in enumerate(self.layers):
            if i == capture_layer:
                boundary = DraftBoundary(h, rotary, allowed, i, past)
            h, kv = layer(h, view, None if cache is None else cache[i], rotary, allowed)
            if view == "ar":
                new_cache.append(kv)
        h = self.norm(h)
        rows = h[:, -logits_to_keep:] if logits_to_keep else h
        logits = self.head(rows) if compute_logits else None
        return BackboneOutput(h, tuple(new_cache) if view == "ar" else cache, logits, boundary)

    def forward_suffix(self, boundary: DraftBoundary, *, cache=None, logit_range=None, draft_weights=None
                       ) -> BackboneOutput:
        """Replay the draft view from a frozen boundary; overrides carry master weights."""
        if cache_length(cache) != boundary.history_length:
            raise ValueError("matching historical cache required")
        overrides = draft_weights or {}
        allowed_keys = {f"layers.{i}.attention.draft.{n}" for i in range(boundary.start_layer, len(self.layers))
                        for n, _ in self.layers[i].attention.draft.named_parameters()}
        if overrides.keys() - allowed_keys:
            raise ValueError("suffix overrides are restricted to draft attention parameters")
        h = boundary.hidden
        for off, layer in enumerate(self.layers[boundary.start_layer:]):
            prefix = f"layers.{boundary.start_layer + off}."
            w = {n[len(prefix):]: v for n, v in overrides.items() if n.startswith(prefix)}
            args = (h, "draft", None if cache is None else cache[off], boundary.rotary, boundary.allowed)
            h, _ = torch.func.functional_call(layer, w, args) if w else layer(*args)
        h = self.norm(h)
        rows = h if logit_range is None else h[:, logit_range[0]:logit_range[1]]
        return BackboneOutput(h, cache, self.head(rows))


def draft_block_mask(history: int, block: int, device) -> Tensor:
    """Draft view mask: the block sees the whole history and itself in both directions."""
    return torch.ones(1, 1, block, history + block, dtype=torch.bool, device=device)
