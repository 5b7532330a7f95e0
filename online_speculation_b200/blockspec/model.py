"""Dual-view decoder: one Qwen3-shaped backbone carrying two attention projection sets.

The ``ar`` view is the ordinary causal decoder and owns the KV history.  The
``draft`` view re-reads that history read-only and attends bidirectionally inside a
block ``[anchor, MASK, ..., MASK]``; embeddings, norms, MLPs and the head are shared.
This module is the PyTorch training / oracle path (distillation, online suffix
replay with :meth:`DualViewDecoder.forward_suffix`, audits); serving on B200 runs the
same weights on the sm_100a kernels (:mod:`online_speculation_b200.blockspec.kernel_branch`).

Attention is computed in fp32 with ``scaled_dot_product_attention`` and grouped KV
heads, under an explicit boolean visibility mask.  Module and parameter names
(``layers.{i}.attention.{ar,draft}.{q,k,v,o,q_norm,k_norm}``, ``input_norm``,
``post_norm``, ``gate``, ``up``, ``down``, ``embedding``, ``norm``, ``head``) are the
state-dict keys of ``blockspec-dual-view-v1`` checkpoints
(online-speculation/src/blockspec/parallel/backbone.py), so checkpoints load unchanged.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, fields

import torch
import torch.nn.functional as F
from torch import Tensor, nn

Cache = tuple  # per layer (k [B, Hkv, T, D], v [B, Hkv, T, D])

VIEWS = ("ar", "draft")


def cache_length(cache) -> int:
    if cache is None:
        return 0
    if not cache:
        raise ValueError("an empty cache is written None, not ()")
    return int(cache[0][0].shape[2])


def trim_cache(cache, length: int):
    """The first ``length`` positions of every layer, detached (None when nothing is left)."""
    if not 0 <= length <= cache_length(cache):
        raise ValueError(f"cannot trim a cache of {cache_length(cache)} positions to {length}")
    if length == 0:
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
        sizes = (self.vocab_size, self.hidden_size, self.intermediate_size, self.num_hidden_layers,
                 self.num_attention_heads, self.num_key_value_heads, self.head_dim)
        checks = (
            (min(sizes) >= 1, "model sizes must be positive"),
            (self.head_dim % 2 == 0, "rotary embeddings need an even head_dim"),
            (self.num_attention_heads % self.num_key_value_heads == 0, "query heads must group evenly over KV heads"),
            (self.block_size >= 2, "a draft block holds the anchor and at least one mask"),
            (0 <= self.mask_token_id < self.vocab_size, "mask_token_id must be a vocabulary id"),
            (self.eos_token_id is None or 0 <= self.eos_token_id < self.vocab_size, "eos_token_id must be a vocabulary id"),
            (math.isfinite(self.rms_norm_eps) and self.rms_norm_eps > 0, "rms_norm_eps must be positive"),
            (math.isfinite(self.rope_theta) and self.rope_theta > 1, "rope_theta must exceed 1"),
        )
        failed = [message for ok, message in checks if not ok]
        if failed:
            raise ValueError("invalid dual-view config: " + "; ".join(failed))

    def to_dict(self) -> dict:
        return asdict(self)

    @classmethod
    def from_public(cls, data: dict) -> "DualViewConfig":
        """From the ``config.json`` of a Qwen3 (or dual-view) checkpoint."""
        rope = data.get("rope_parameters") or data.get("rope_scaling") or {}
        problems = []
        if data.get("model_type") not in ("qwen3", "orthrus"):
            problems.append("model_type must be qwen3")
        if data.get("hidden_act", "silu") != "silu":
            problems.append("the MLP must be SwiGLU (hidden_act silu)")
        if data.get("use_sliding_window", False) or set(data.get("layer_types", [])) - {"full_attention"}:
            problems.append("only full attention is implemented")
        if rope.get("rope_type", rope.get("type", "default")) != "default":
            problems.append("only plain RoPE is implemented")
        if problems:
            raise ValueError("cannot import this checkpoint: " + "; ".join(problems))
        names = [f.name for f in fields(cls)]
        values = {k: data[k] for k in names if k in data}
        if "rope_theta" in rope:
            values["rope_theta"] = rope["rope_theta"]
        optional = {"attention_bias", "tie_word_embeddings", "eos_token_id"}
        missing = sorted(set(names) - optional - set(values))
        if missing:
            raise ValueError(f"config.json lacks architecture fields {missing}")
        return cls(**values)


class RMSNorm(nn.Module):
    def __init__(self, width: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.epsilon = eps

    def forward(self, x: Tensor) -> Tensor:
        x32 = x.float()
        scale = torch.rsqrt(x32.pow(2).mean(dim=-1, keepdim=True) + self.epsilon)
        return (x32 * scale).to(x.dtype) * self.weight


def rotate(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    """Rotate-half RoPE: pairs (i, i + D/2) turn by the position's angle."""
    first, second = x.chunk(2, dim=-1)
    turned = torch.cat((-second, first), dim=-1)
    return x * cos + turned * sin


class AttentionView(nn.Module):
    """One projection set (q, k, v, o) with per-head Q / K RMSNorm."""

    def __init__(self, c: DualViewConfig):
        super().__init__()
        q_width = c.num_attention_heads * c.head_dim
        kv_width = c.num_key_value_heads * c.head_dim
        self.q = nn.Linear(c.hidden_size, q_width, bias=c.attention_bias)
        self.k = nn.Linear(c.hidden_size, kv_width, bias=c.attention_bias)
        self.v = nn.Linear(c.hidden_size, kv_width, bias=c.attention_bias)
        self.o = nn.Linear(q_width, c.hidden_size, bias=c.attention_bias)
        self.q_norm = RMSNorm(c.head_dim, c.rms_norm_eps)
        self.k_norm = RMSNorm(c.head_dim, c.rms_norm_eps)
        self.head_dim = c.head_dim

    def heads(self, x: Tensor, rotary) -> tuple[Tensor, Tensor, Tensor]:
        """q [B, Hq, T, D], k and v [B, Hkv, T, D] with Q/K norm and RoPE applied."""
        B, T, _ = x.shape
        split = lambda t: t.view(B, T, -1, self.head_dim).transpose(1, 2)   # noqa: E731
        cos, sin = rotary
        q = rotate(split(self.q_norm(self.q(x).view(B, T, -1, self.head_dim)).flatten(2)), cos, sin)
        k = rotate(split(self.k_norm(self.k(x).view(B, T, -1, self.head_dim)).flatten(2)), cos, sin)
        return q, k, split(self.v(x))


class DualAttention(nn.Module):
    def __init__(self, c: DualViewConfig):
        super().__init__()
        self.config = c
        self.ar = AttentionView(c)
        self.draft = AttentionView(c)

    def forward(self, x, view, cache, rotary, allowed):
        projections: AttentionView = getattr(self, view)
        q, k, v = projections.heads(x, rotary)
        if cache is not None:
            k = torch.cat((cache[0], k), dim=2)
            v = torch.cat((cache[1], v), dim=2)
        mixed = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=allowed,
                                               enable_gqa=q.shape[1] != k.shape[1])
        B, _, T, _ = q.shape
        return projections.o(mixed.to(q.dtype).transpose(1, 2).reshape(B, T, -1)), (k, v)


class DualLayer(nn.Module):
    def __init__(self, c: DualViewConfig):
        super().__init__()
        self.attention = DualAttention(c)
        self.input_norm = RMSNorm(c.hidden_size, c.rms_norm_eps)
        self.post_norm = RMSNorm(c.hidden_size, c.rms_norm_eps)
        self.gate = nn.Linear(c.hidden_size, c.intermediate_size, bias=False)
        self.up = nn.Linear(c.hidden_size, c.intermediate_size, bias=False)
        self.down = nn.Linear(c.intermediate_size, c.hidden_size, bias=False)

    def _mlp(self, x: Tensor) -> Tensor:
        n = self.post_norm(x)
        return self.down(F.silu(self.gate(n)) * self.up(n))

    def forward(self, x, view, cache, rotary, allowed):
        mixed, kv = self.attention(self.input_norm(x), view, cache, rotary, allowed)
        x = x + mixed
        return x + self._mlp(x), kv


@dataclass
class DraftBoundary:
    """Input of the first replayed layer, frozen for online suffix replay."""

    hidden: Tensor
    rotary: tuple
    allowed: Tensor | None
    start_layer: int
    history_length: int

    def detached(self) -> "DraftBoundary":
        copy = lambda t: t.detach().clone()   # noqa: E731
        return DraftBoundary(copy(self.hidden), tuple(map(copy, self.rotary)),
                             None if self.allowed is None else copy(self.allowed), self.start_layer,
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
        self.layers = nn.ModuleList([DualLayer(config) for _ in range(config.num_hidden_layers)])
        self.norm = RMSNorm(config.hidden_size, config.rms_norm_eps)
        self.head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        self.register_buffer("frequencies", self._frequencies(self.embedding.weight.device), persistent=False)
        self._init_weights()
        self.tie_weights()
        self.initialize_draft_from_ar()
        self.source: dict = {}

    def _init_weights(self) -> None:
        for module in self.modules():
            if isinstance(module, (nn.Linear, nn.Embedding)):
                nn.init.normal_(module.weight, std=0.02)
            if isinstance(module, nn.Linear) and module.bias is not None:
                nn.init.zeros_(module.bias)

    def tie_weights(self):
        if self.config.tie_word_embeddings:
            self.head.weight = self.embedding.weight

    def _frequencies(self, device):
        # built in fp32 on the host, then moved
        exponents = torch.arange(0, self.config.head_dim, 2, dtype=torch.float32) / self.config.head_dim
        return torch.pow(self.config.rope_theta, -exponents).to(device)

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
        angles = positions.float().unsqueeze(-1) * self.frequencies
        angles = angles.repeat(*([1] * (angles.ndim - 1)), 2).unsqueeze(1)
        return angles.cos().to(dtype), angles.sin().to(dtype)

    @staticmethod
    def _causal(past: int, T: int, device) -> Tensor:
        queries = torch.arange(past, past + T, device=device)
        keys = torch.arange(past + T, device=device)
        return (keys.unsqueeze(0) <= queries.unsqueeze(1)).unsqueeze(0).unsqueeze(0)

    def forward(self, tokens: Tensor, *, view: str = "ar", cache=None, positions=None, allowed=None,
                logits_to_keep: int = 0, compute_logits: bool = True, capture_layer: int | None = None
                ) -> BackboneOutput:
        if view not in VIEWS:
            raise ValueError(f"view {view!r} is not one of {VIEWS}")
        if tokens.ndim != 2 or tokens.shape[1] == 0:
            raise ValueError("tokens must be a non-empty [batch, time] tensor")
        if capture_layer is not None and not (view == "draft" and 0 <= capture_layer < len(self.layers)):
            raise ValueError("a boundary is captured only in the draft view, at an existing layer")
        T = tokens.shape[1]
        past = cache_length(cache)
        if positions is None:
            positions = torch.arange(past, past + T, device=tokens.device).unsqueeze(0)
        if allowed is None and view == "ar":
            allowed = self._causal(past, T, tokens.device)
        h = self.embedding(tokens)
        rotary = self._rotary(positions, h.dtype)
        written, boundary = [], None
        for i, layer in enumerate(self.layers):
            if i == capture_layer:
                boundary = DraftBoundary(h, rotary, allowed, i, past)
            h, kv = layer(h, view, None if cache is None else cache[i], rotary, allowed)
            written.append(kv)
        h = self.norm(h)
        logits = None
        if compute_logits:
            logits = self.head(h[:, -logits_to_keep:] if logits_to_keep else h)
        # the draft view reads the history but never extends it
        return BackboneOutput(h, tuple(written) if view == "ar" else cache, logits, boundary)

    def forward_suffix(self, boundary: DraftBoundary, *, cache=None, logit_range=None, draft_weights=None
                       ) -> BackboneOutput:
        """Replay the draft view from a frozen boundary; overrides supply master draft weights."""
        if cache_length(cache) != boundary.history_length:
            raise ValueError("the replay needs the cache the boundary was captured with")
        overrides = dict(draft_weights or {})
        start = boundary.start_layer
        replayed = list(enumerate(self.layers))[start:]
        legal = {f"layers.{i}.attention.draft.{name}" for i, layer in replayed
                 for name, _ in layer.attention.draft.named_parameters()}
        if set(overrides) - legal:
            raise ValueError("suffix overrides may only replace draft attention parameters of replayed layers")
        h = boundary.hidden
        for offset, (i, layer) in enumerate(replayed):
            prefix = f"layers.{i}."
            local = {name[len(prefix):]: value for name, value in overrides.items() if name.startswith(prefix)}
            args = (h, "draft", None if cache is None else cache[offset], boundary.rotary, boundary.allowed)
            h, _ = torch.func.functional_call(layer, local, args) if local else layer(*args)
        h = self.norm(h)
        rows = h if logit_range is None else h[:, logit_range[0]:logit_range[1]]
        return BackboneOutput(h, cache, self.head(rows))


def draft_block_mask(history: int, block: int, device) -> Tensor:
    """Draft view visibility: every block row sees the whole history and the whole block."""
    return torch.ones(1, 1, block, history + block, dtype=torch.bool, device=device)
