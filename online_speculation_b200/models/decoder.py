"""Qwen2 / Qwen3-shaped causal decoders laid out for the sm_100a kernels.

One :class:`DecoderConfig` covers the reference's autoregressive models: the
Qwen2.5 decoders driven through HF Transformers by
src/inference_scaling/arllm/backends/transformers_backend.py (GQA, RoPE
theta 1e6, SwiGLU, QKV bias) and the Qwen3-shaped backbone of
online-speculation/src/blockspec/parallel/backbone.py:15-71 (per-head Q/K
RMSNorm, no bias, tied embeddings).

Weights are stored per tensor-parallel rank in the fused layouts the kernels
consume:

* ``w_qkv``  [(q_slots + 2 * kv_slots) * D, H]  (column parallel, with bias)
* ``w_o``    [H, q_slots * D]                   (row parallel)
* ``w_gu``   [2 * F_local, H]  tiles of [64 gate rows | 64 up rows]
* ``w_down`` [H, F_local]                        (row parallel)
* ``head``   [V_local, H]                        (vocabulary parallel)

Query heads that do not divide evenly over the ranks (28 heads on 8 GPUs)
are padded with zero heads so that every rank holds the same number of query
slots, each rank's slots map to one KV head group, and a KV head is replicated
on the ranks that share it.  Padded slots have zero Q and O weights and add
nothing to the output.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import torch

from ..ops import kernels as K

HEAD_DIM = 128


@dataclass(frozen=True)
class DecoderConfig:
    vocab_size: int = 151936
    hidden_size: int = 1536
    intermediate_size: int = 8960
    num_hidden_layers: int = 28
    num_attention_heads: int = 12
    num_key_value_heads: int = 2
    head_dim: int = HEAD_DIM
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    attention_bias: bool = True
    qk_norm: bool = False
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 32768
    eos_token_id: int | None = None
    name: str = "decoder"

    def __post_init__(self):
        if self.head_dim != HEAD_DIM:
            raise ValueError("the attention kernels are built for head_dim 128")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        if self.hidden_size % 8:
            raise ValueError("hidden size must be a multiple of 8")

    @property
    def group(self) -> int:
        return self.num_attention_heads // self.num_key_value_heads

    def parameter_count(self) -> int:
        H, F, V, L = self.hidden_size, self.intermediate_size, self.vocab_size, self.num_hidden_layers
        q, kv = self.num_attention_heads * self.head_dim, self.num_key_value_heads * self.head_dim
        per_layer = H * (q + 2 * kv) + q * H + 3 * H * F + 2 * H
        if self.attention_bias:
            per_layer += q + 2 * kv
        head = 0 if self.tie_word_embeddings else V * H
        return L * per_layer + V * H + head + H

    def to_dict(self):
        return asdict(self)

    @classmethod
    def from_hf(cls, data: dict, name: str = "hf") -> "DecoderConfig":
        """Build from a HF ``config.json`` dictionary of a Qwen2 / Qwen3 model."""
        model_type = data.get("model_type", "qwen2")
        if model_type not in ("qwen2", "qwen3"):
            raise ValueError(f"unsupported model_type {model_type!r}")
        if data.get("hidden_act", "silu") != "silu":
            raise ValueError("SwiGLU activation required")
        rope = data.get("rope_parameters") or data.get("rope_scaling") or {}
        theta = rope.get("rope_theta", data.get("rope_theta", 1_000_000.0))
        heads = data["num_attention_heads"]
        return cls(vocab_size=data["vocab_size"], hidden_size=data["hidden_size"],
                   intermediate_size=data["intermediate_size"], num_hidden_layers=data["num_hidden_layers"],
                   num_attention_heads=heads, num_key_value_heads=data.get("num_key_value_heads", heads),
                   head_dim=data.get("head_dim", data["hidden_size"] // heads), rope_theta=float(theta),
                   rms_norm_eps=data.get("rms_norm_eps", 1e-6),
                   attention_bias=data.get("attention_bias", model_type == "qwen2"), qk_norm=model_type == "qwen3",
                   tie_word_embeddings=data.get("tie_word_embeddings", False),
                   max_position_embeddings=data.get("max_position_embeddings", 32768),
                   eos_token_id=data.get("eos_token_id") if isinstance(data.get("eos_token_id"), int) else None,
                   name=name)


PRESETS = {
    "qwen2.5-0.5b": DecoderConfig(vocab_size=151936, hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                                  num_attention_heads=14, num_key_value_heads=2, tie_word_embeddings=True,
                                  name="qwen2.5-0.5b"),
    "qwen2.5-1.5b": DecoderConfig(vocab_size=151936, hidden_size=1536, intermediate_size=8960, num_hidden_layers=28,
                                  num_attention_heads=12, num_key_value_heads=2, tie_word_embeddings=True,
                                  name="qwen2.5-1.5b"),
    "qwen2.5-7b": DecoderConfig(vocab_size=152064, hidden_size=3584, intermediate_size=18944, num_hidden_layers=28,
                                num_attention_heads=28, num_key_value_heads=4, name="qwen2.5-7b"),
    "qwen3-1.7b": DecoderConfig(vocab_size=151936, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                                num_attention_heads=16, num_key_value_heads=8, attention_bias=False, qk_norm=True,
                                tie_word_embeddings=True, name="qwen3-1.7b"),
    "tiny": DecoderConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                          num_attention_heads=4, num_key_value_heads=2, name="tiny"),
}


@dataclass(frozen=True)
class HeadLayout:
    """Assignment of query / KV heads to one tensor-parallel rank.

    ``q_heads``: global query head of every local slot (-1 = zero padding).
    ``kv_heads``: global KV head of every local KV slot.
    Local query slot s uses local KV slot s // (q_slots // kv_slots).
    """

    q_heads: tuple[int, ...]
    kv_heads: tuple[int, ...]

    @property
    def q_slots(self) -> int:
        return len(self.q_heads)

    @property
    def kv_slots(self) -> int:
        return len(self.kv_heads)


def head_layout(num_q: int, num_kv: int, tp: int, rank: int) -> HeadLayout:
    group = num_q // num_kv
    if tp <= num_kv:
        if num_kv % tp:
            raise ValueError(f"{num_kv} KV heads cannot be split over {tp} ranks")
        kv = list(range(rank * num_kv // tp, (rank + 1) * num_kv // tp))
        q = [h for g in kv for h in range(g * group, (g + 1) * group)]
        return HeadLayout(tuple(q), tuple(kv))
    if tp % num_kv:
        raise ValueError(f"{tp} ranks cannot share {num_kv} KV heads evenly")
    share = tp // num_kv            # ranks per KV head
    g = rank // share
    part = rank % share
    per = -(-group // share)        # query slots per rank (ceil)
    heads = [g * group + i for i in range(part * per, min(group, (part + 1) * per))]
    heads += [-1] * (per - len(heads))
    return HeadLayout(tuple(heads), (g,))


def _shard_rows(n: int, tp: int, rank: int, multiple: int = 1) -> tuple[int, int]:
    per = -(-n // (tp * multiple)) * multiple
    lo = min(n, rank * per)
    return lo, min(n, lo + per)


@dataclass
class LayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    w_qkv: torch.Tensor
    b_qkv: torch.Tensor | None
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    w_o: torch.Tensor
    w_gu: torch.Tensor
    w_down: torch.Tensor


@dataclass
class DecoderWeights:
    """One rank's weights in kernel layout plus the layout metadata."""

    config: DecoderConfig
    tp: int
    rank: int
    heads: HeadLayout
    ffn_local: int             # padded local intermediate width (multiple of 64)
    vocab_range: tuple[int, int]
    embed: torch.Tensor        # [V, H] replicated
    final_norm: torch.Tensor
    head: torch.Tensor         # [V_local, H]
    layers: list[LayerWeights] = field(default_factory=list)
    inv_freq: torch.Tensor | None = None

    @property
    def device(self) -> torch.device:
        return self.embed.device

    def nbytes(self) -> int:
        total = self.embed.numel() + self.head.numel()
        for lw in self.layers:
            total += sum(t.numel() for t in (lw.w_qkv, lw.w_o, lw.w_gu, lw.w_down))
        return 2 * total


def build_weights(config: DecoderConfig, full: dict[str, torch.Tensor], *, tp: int = 1, rank: int = 0,
                  device="cpu", dtype=torch.bfloat16) -> DecoderWeights:
    """Shard a full HF-named state dict into one rank's kernel layout."""
    D, H = config.head_dim, config.hidden_size
    layout = head_layout(config.num_attention_heads, config.num_key_value_heads, tp, rank)
    f_lo, f_hi = _shard_rows(config.intermediate_size, tp, rank, 64)
    ffn_local = -(-config.intermediate_size // (tp * 64)) * 64   # equal padded width on every rank
    v_lo, v_hi = _shard_rows(config.vocab_size, tp, rank)

    def get(name):
        t = full[name]
        return t.to(dtype) if t.is_floating_point() else t

    def heads_rows(t, heads, width=D):
        # select per-head row blocks; -1 -> zeros
        blocks = [t[h * width:(h + 1) * width] if h >= 0 else torch.zeros_like(t[:width]) for h in heads]
        return torch.cat(blocks, 0)

    def heads_cols(t, heads, width=D):
        blocks = [t[:, h * width:(h + 1) * width] if h >= 0 else torch.zeros_like(t[:, :width]) for h in heads]
        return torch.cat(blocks, 1)

    embed = get("model.embed_tokens.weight")
    head_full = embed if config.tie_word_embeddings else get("lm_head.weight")
    weights = DecoderWeights(config, tp, rank, layout, ffn_local, (v_lo, v_hi), embed.to(device).contiguous(),
                             get("model.norm.weight").to(device).contiguous(),
                             head_full[v_lo:v_hi].to(device).contiguous())
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        q = heads_rows(get(p + "self_attn.q_proj.weight"), layout.q_heads)
        k = heads_rows(get(p + "self_attn.k_proj.weight"), layout.kv_heads)
        v = heads_rows(get(p + "self_attn.v_proj.weight"), layout.kv_heads)
        bias = None
        if config.attention_bias:
            bias = torch.cat((heads_rows(get(p + "self_attn.q_proj.bias"), layout.q_heads),
                              heads_rows(get(p + "self_attn.k_proj.bias"), layout.kv_heads),
                              heads_rows(get(p + "self_attn.v_proj.bias"), layout.kv_heads)))
        o = heads_cols(get(p + "self_attn.o_proj.weight"), layout.q_heads)
        gate = get(p + "mlp.gate_proj.weight")[f_lo:f_hi]
        up = get(p + "mlp.up_proj.weight")[f_lo:f_hi]
        down = get(p + "mlp.down_proj.weight")[:, f_lo:f_hi]
        pad = ffn_local - gate.shape[0]
        if pad:
            gate = torch.cat((gate, gate.new_zeros(pad, H)))
            up = torch.cat((up, up.new_zeros(pad, H)))
            down = torch.cat((down, down.new_zeros(H, pad)), 1)
        lw = LayerWeights(
            get(p + "input_layernorm.weight").to(device).contiguous(),
            get(p + "post_attention_layernorm.weight").to(device).contiguous(),
            torch.cat((q, k, v)).to(device).contiguous(),
            None if bias is None else bias.to(device).contiguous(),
            get(p + "self_attn.q_norm.weight").to(device).contiguous() if config.qk_norm else None,
            get(p + "self_attn.k_norm.weight").to(device).contiguous() if config.qk_norm else None,
            o.to(device).contiguous(),
            K.interleave_gate_up(gate, up).to(device),
            down.to(device).contiguous(),
        )
        weights.layers.append(lw)
    weights.inv_freq = K.rope_frequencies(D, config.rope_theta).to(device)
    return weights


def random_state_dict(config: DecoderConfig, *, seed: int = 0, std: float = 0.02, device="cpu",
                      dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Random-init HF-named weights (normal(0, std) matrices, unit norms, zero bias)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, F, V = config.hidden_size, config.intermediate_size, config.vocab_size
    q, kv = config.num_attention_heads * config.head_dim, config.num_key_value_heads * config.head_dim

    def mat(rows, cols):
        return (torch.randn(rows, cols, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

    sd = {"model.embed_tokens.weight": mat(V, H), "model.norm.weight": torch.ones(H, dtype=dtype, device=device)}
    if not config.tie_word_embeddings:
        sd["lm_head.weight"] = mat(V, H)
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = mat(q, H)
        sd[p + "self_attn.k_proj.weight"] = mat(kv, H)
        sd[p + "self_attn.v_proj.weight"] = mat(kv, H)
        sd[p + "self_attn.o_proj.weight"] = mat(H, q)
        if config.attention_bias:
            for n, w in (("q", q), ("k", kv), ("v", kv)):
                sd[p + f"self_attn.{n}_proj.bias"] = torch.zeros(w, dtype=dtype, device=device)
        if config.qk_norm:
            sd[p + "self_attn.q_norm.weight"] = torch.ones(config.head_dim, dtype=dtype, device=device)
            sd[p + "self_attn.k_norm.weight"] = torch.ones(config.head_dim, dtype=dtype, device=device)
        sd[p + "mlp.gate_proj.weight"] = mat(F, H)
        sd[p + "mlp.up_proj.weight"] = mat(F, H)
        sd[p + "mlp.down_proj.weight"] = mat(H, F)
        sd[p + "input_layernorm.weight"] = torch.ones(H, dtype=dtype, device=device)
        sd[p + "post_attention_layernorm.weight"] = torch.ones(H, dtype=dtype, device=device)
    return sd


def random_weights(config: DecoderConfig, *, tp: int = 1, rank: int = 0, seed: int = 0, device="cuda",
                   std: float = 0.02) -> DecoderWeights:
    """Random-init weights built directly for one rank (avoids materialising the full model per rank).

    Every rank draws the same full matrices from the same seed on the device and
    keeps its shard, so shards agree with a single-GPU model of the same seed.
    """
    sd = random_state_dict(config, seed=seed, std=std, device=device)
    w = build_weights(config, sd, tp=tp, rank=rank, device=device)
    del sd
    return w


# ------------------------------------------------------------ fp32 oracle --
def reference_forward(config: DecoderConfig, sd: dict[str, torch.Tensor], tokens: torch.Tensor) -> torch.Tensor:
    """Plain fp32 PyTorch forward of a full HF-named state dict: logits [T, V] of one causal sequence."""
    D = config.head_dim
    f = {k: v.float() for k, v in sd.items()}
    x = f["model.embed_tokens.weight"][tokens.long()]
    T = x.shape[0]
    pos = torch.arange(T, dtype=torch.float32)
    inv = K.rope_frequencies(D, config.rope_theta)
    ang = pos[:, None] * inv[None]
    cos, sin = ang.cos(), ang.sin()

    def norm(h, w, eps=config.rms_norm_eps):
        return h * torch.rsqrt(h.square().mean(-1, keepdim=True) + eps) * w

    def rope(t):
        a, b = t[..., : D // 2], t[..., D // 2:]
        c, s = cos[:, None], sin[:, None]
        return torch.cat((a * c - b * s, b * c + a * s), -1)

    mask = torch.ones(T, T, dtype=torch.bool).tril()
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        h = norm(x, f[p + "input_layernorm.weight"])
        q = h @ f[p + "self_attn.q_proj.weight"].t()
        k = h @ f[p + "self_attn.k_proj.weight"].t()
        v = h @ f[p + "self_attn.v_proj.weight"].t()
        if config.attention_bias:
            q, k, v = q + f[p + "self_attn.q_proj.bias"], k + f[p + "self_attn.k_proj.bias"], v + f[
                p + "self_attn.v_proj.bias"]
        q = q.view(T, -1, D)
        k = k.view(T, -1, D)
        v = v.view(T, -1, D)
        if config.qk_norm:
            q = norm(q, f[p + "self_attn.q_norm.weight"])
            k = norm(k, f[p + "self_attn.k_norm.weight"])
        q, k = rope(q), rope(k)
        k = k.repeat_interleave(config.group, 1)
        v = v.repeat_interleave(config.group, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(D)
        s = s.masked_fill(~mask, float("-inf"))
        a = torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(T, -1)
        x = x + a @ f[p + "self_attn.o_proj.weight"].t()
        h = norm(x, f[p + "post_attention_layernorm.weight"])
        gate = h @ f[p + "mlp.gate_proj.weight"].t()
        up = h @ f[p + "mlp.up_proj.weight"].t()
        x = x + (torch.nn.functional.silu(gate) * up) @ f[p + "mlp.down_proj.weight"].t()
    x = norm(x, f["model.norm.weight"])
    head = f["model.embed_tokens.weight"] if config.tie_word_embeddings else f["lm_head.weight"]
    return x @ head.t()
