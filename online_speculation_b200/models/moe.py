"""LLaDA-MoE-shaped masked-diffusion decoder on the sm_100a kernels.

The reference runs LLaDA-MoE-7B-A1B through HF remote code
(src/inference_scaling/dllm/backends/llada.py:417-448 calls the model on the
full sequence every reverse step; MoE parameters are counted at :347-370).
This module is the same network shape built for B200:

* bidirectional attention over the whole sequence (no KV cache across steps:
  K/V of a layer are written to a one-layer paged scratch and consumed by the
  paged attention kernel in bidirectional mode right away);
* per-head Q/K RMSNorm and RoPE fused in one kernel;
* MoE FFN: router GEMM, on-device top-k routing and dispatch, grouped tcgen05
  GEMMs over all experts (SwiGLU fused), weighted combine into the residual
  stream (``ops.kernels.moe_ffn``);
* logits only for the rows the sampler needs (the current block), never for
  every position.

Weights in kernel layout: ``w_qkv`` [3 * heads * D, H]; ``w_o`` [H, heads * D];
``router`` [E, H]; ``w_gu`` [E * 2F, H] (each expert's gate / up rows
interleaved in 64-row tiles); ``w_down`` [E * H, F].
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field

import torch

from ..ops import kernels as K

PAGE = 32


@dataclass(frozen=True)
class MoEConfig:
    vocab_size: int = 157184
    hidden_size: int = 2048
    num_hidden_layers: int = 16
    num_attention_heads: int = 16
    num_key_value_heads: int = 16
    head_dim: int = 128
    num_experts: int = 64
    num_experts_per_tok: int = 8
    moe_intermediate_size: int = 1024
    norm_topk_prob: bool = False
    rope_theta: float = 50000.0
    rms_norm_eps: float = 1e-6
    qk_norm: bool = True
    tie_word_embeddings: bool = False
    mask_token_id: int = 156895
    name: str = "moe"

    def __post_init__(self):
        if self.head_dim != 128:
            raise ValueError("the attention kernels are built for head_dim 128")
        if self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("query heads must be a multiple of KV heads")
        if self.hidden_size % 128 or (2 * self.moe_intermediate_size) % 128:
            raise ValueError("hidden and expert widths must be multiples of 64 (gate/up tiles) / 128")
        if not 0 < self.num_experts_per_tok <= min(self.num_experts, 32) or self.num_experts > 256:
            raise ValueError("top-k must lie in [1, min(E, 32)] with at most 256 experts")
        if not 0 <= self.mask_token_id < self.vocab_size:
            raise ValueError("mask_token_id must be a vocabulary id")

    def parameter_counts(self) -> tuple[int, int]:
        """(total, active per token) parameters."""
        H, D, V = self.hidden_size, self.head_dim, self.vocab_size
        att = H * (self.num_attention_heads + 2 * self.num_key_value_heads) * D + self.num_attention_heads * D * H
        expert = 3 * H * self.moe_intermediate_size
        per_layer_shared = att + self.num_experts * H + 2 * H
        head = 0 if self.tie_word_embeddings else V * H
        total = self.num_hidden_layers * (per_layer_shared + self.num_experts * expert) + V * H + head + H
        active = self.num_hidden_layers * (per_layer_shared + self.num_experts_per_tok * expert) + V * H + head + H
        return total, active

    def to_dict(self):
        return asdict(self)


PRESETS = {
    "llada-moe-7b-a1b": MoEConfig(name="llada-moe-7b-a1b"),
    "tiny-moe": MoEConfig(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=2,
                          num_key_value_heads=2, num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
                          mask_token_id=511, name="tiny-moe"),
}


def random_state_dict(config: MoEConfig, *, seed: int = 0, std: float = 0.02, device="cpu",
                      dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Random-init weights with HF-style names (OLMoE / LLaDA-MoE layout)."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, V, D = config.hidden_size, config.vocab_size, config.head_dim
    q, kv, F = config.num_attention_heads * D, config.num_key_value_heads * D, config.moe_intermediate_size

    def mat(rows, cols):
        return (torch.randn(rows, cols, generator=g, device=device, dtype=torch.float32) * std).to(dtype)

    def ones(n):
        return torch.ones(n, dtype=dtype, device=device)

    sd = {"model.embed_tokens.weight": mat(V, H), "model.norm.weight": ones(H)}
    if not config.tie_word_embeddings:
        sd["lm_head.weight"] = mat(V, H)
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        sd[p + "self_attn.q_proj.weight"] = mat(q, H)
        sd[p + "self_attn.k_proj.weight"] = mat(kv, H)
        sd[p + "self_attn.v_proj.weight"] = mat(kv, H)
        sd[p + "self_attn.o_proj.weight"] = mat(H, q)
        if config.qk_norm:
            sd[p + "self_attn.q_norm.weight"] = ones(D)
            sd[p + "self_attn.k_norm.weight"] = ones(D)
        sd[p + "mlp.gate.weight"] = mat(config.num_experts, H)
        for e in range(config.num_experts):
            sd[p + f"mlp.experts.{e}.gate_proj.weight"] = mat(F, H)
            sd[p + f"mlp.experts.{e}.up_proj.weight"] = mat(F, H)
            sd[p + f"mlp.experts.{e}.down_proj.weight"] = mat(H, F)
        sd[p + "input_layernorm.weight"] = ones(H)
        sd[p + "post_attention_layernorm.weight"] = ones(H)
    return sd


@dataclass
class MoELayerWeights:
    in_norm: torch.Tensor
    post_norm: torch.Tensor
    w_qkv: torch.Tensor
    q_norm: torch.Tensor | None
    k_norm: torch.Tensor | None
    w_o: torch.Tensor
    router: torch.Tensor
    w_gu: torch.Tensor      # [E_local * 2F, H]
    w_down: torch.Tensor    # [E_local * H, F]


@dataclass
class MoEWeights:
    config: MoEConfig
    embed: torch.Tensor
    final_norm: torch.Tensor
    head: torch.Tensor
    layers: list[MoELayerWeights] = field(default_factory=list)
    inv_freq: torch.Tensor | None = None
    expert_range: tuple[int, int] = (0, 0)   # experts held by this rank (expert parallelism)


def build_weights(config: MoEConfig, sd: dict[str, torch.Tensor], *, device="cpu", dtype=torch.bfloat16,
                  expert_range: tuple[int, int] | None = None) -> MoEWeights:
    """HF-named weights -> kernel layout (optionally only the experts in ``expert_range``)."""
    lo, hi = expert_range or (0, config.num_experts)

    def get(name):
        return sd[name].to(device=device, dtype=dtype).contiguous()

    embed = get("model.embed_tokens.weight")
    head = embed if config.tie_word_embeddings else get("lm_head.weight")
    w = MoEWeights(config, embed, get("model.norm.weight"), head, expert_range=(lo, hi))
    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        qkv = torch.cat([get(p + f"self_attn.{n}_proj.weight") for n in ("q", "k", "v")]).contiguous()
        gu = torch.cat([K.interleave_gate_up(get(p + f"mlp.experts.{e}.gate_proj.weight"),
                                             get(p + f"mlp.experts.{e}.up_proj.weight")) for e in range(lo, hi)])
        down = torch.cat([get(p + f"mlp.experts.{e}.down_proj.weight") for e in range(lo, hi)])
        w.layers.append(MoELayerWeights(
            get(p + "input_layernorm.weight"), get(p + "post_attention_layernorm.weight"), qkv,
            get(p + "self_attn.q_norm.weight") if config.qk_norm else None,
            get(p + "self_attn.k_norm.weight") if config.qk_norm else None,
            get(p + "self_attn.o_proj.weight"), get(p + "mlp.gate.weight"), gu.contiguous(), down.contiguous()))
    w.inv_freq = K.rope_frequencies(config.head_dim, config.rope_theta).to(device)
    return w


class MoEDiffusionModel:
    """Bidirectional MoE decoder; ``logits(tokens, rows)`` returns fp32 logits of the requested rows.

    ``tokens`` [B, L] int; ``rows`` [B, R] int positions (the same R for every
    sequence) or None for all positions.  Buffers are sized lazily and kept.
    """

    def __init__(self, weights: MoEWeights, *, ep=None):
        self.w = weights
        self.cfg = weights.config
        self.device = weights.embed.device
        self.ep = ep                      # expert-parallel dispatcher (parallel.ep), None = all experts local
        self._bufs: dict = {}
        self._moe_buf = None
        self.forward_calls = 0
        self.token_slots = 0

    @property
    def vocab_size(self) -> int:
        return self.cfg.vocab_size

    @property
    def mask_token_id(self) -> int:
        return self.cfg.mask_token_id

    def _buf(self, name, shape, dtype=torch.bfloat16):
        n = math.prod(shape)
        b = self._bufs.get(name)
        if b is None or b.numel() < n or b.dtype != dtype:
            b = torch.empty(n, dtype=dtype, device=self.device)
            self._bufs[name] = b
        return b[:n].view(*shape)

    def _layout(self, B: int, L: int):
        key = (B, L)
        lay = self._bufs.get(("layout", key))
        if lay is None:
            pps = -(-L // PAGE)
            dev = self.device
            table = (torch.arange(B, dtype=torch.int32)[:, None] * pps + torch.arange(pps, dtype=torch.int32)[None])
            pos = torch.arange(L, dtype=torch.int32).repeat(B)
            slots = (torch.arange(B, dtype=torch.int32)[:, None] * (pps * PAGE)
                     + torch.arange(L, dtype=torch.int32)[None]).reshape(-1)
            G = self.cfg.num_attention_heads // self.cfg.num_key_value_heads
            plan = K.plan_attention(table, [L] * B, [L] * B, [1] * B, G, dev, kv_heads=self.cfg.num_key_value_heads)
            lay = (pos.to(dev), slots.to(dev), plan, B * pps)
            self._bufs[("layout", key)] = lay
        return lay

    def hidden(self, tokens: torch.Tensor, layer_limit: int | None = None) -> torch.Tensor:
        """Final residual stream [B * L, H] (before the final norm) after the first ``layer_limit`` layers."""
        c = self.cfg
        B, L = tokens.shape
        T = B * L
        H, D = c.hidden_size, c.head_dim
        nq, nkv = c.num_attention_heads, c.num_key_value_heads
        ids = tokens.reshape(-1).to(device=self.device, dtype=torch.int32)
        pos, slots, plan, pages = self._layout(B, L)
        h = self._buf("h", (T, H))
        x = self._buf("x", (T, H))
        qkv = self._buf("qkv", (T, (nq + 2 * nkv) * D))
        q = self._buf("q", (T, nq, D))
        att = self._buf("att", (T, nq, D))
        kc = self._buf("kc", (pages, nkv, PAGE, D))
        vc = self._buf("vc", (pages, nkv, PAGE, D))
        if self._moe_buf is None or self._moe_buf.T < T:
            self._moe_buf = K.MoEBuffers(T, c.num_experts, c.num_experts_per_tok, H, c.moe_intermediate_size,
                                         self.device) if self.device.type == "cuda" else None
        K.embed(ids, self.w.embed, out=h)
        layers = self.w.layers if layer_limit is None else self.w.layers[:layer_limit]
        if self.ep is not None and layer_limit is not None:
            raise ValueError("an expert-parallel model runs every layer on every rank")
        for lw in layers:
            K.rmsnorm(h, lw.in_norm, c.rms_norm_eps, out=x)
            K.linear(x, lw.w_qkv, out=qkv, static_weights=True)
            K.rope_cache(qkv, pos, slots, self.w.inv_freq, q, kc, vc, nq, nkv, q_norm=lw.q_norm, k_norm=lw.k_norm,
                         eps=c.rms_norm_eps)
            K.attention(q, kc, vc, plan, out=att)
            K.linear(att.view(T, -1), lw.w_o, residual=h, out=h, static_weights=True)
            K.rmsnorm(h, lw.post_norm, c.rms_norm_eps, out=x)
            if self.ep is not None:
                self.ep.moe_ffn(x, h, lw, c)
            else:
                K.moe_ffn(x, h, lw.router, lw.w_gu, lw.w_down, top_k=c.num_experts_per_tok,
                          renorm=c.norm_topk_prob, buffers=self._moe_buf)
        self.forward_calls += 1
        self.token_slots += T
        return h

    # logits(guidance=s) applies classifier-free guidance before the head (see below)
    hidden_guidance = True

    def logits(self, tokens: torch.Tensor, rows: torch.Tensor | None = None,
               layer_limit: int | None = None, *, guidance: float = 0.0) -> torch.Tensor:
        """fp32 logits of ``rows`` (all positions when None).

        ``guidance`` = s > 0: ``tokens`` / ``rows`` stack B conditional and then
        B unconditional sequences, and the result is the B guided rows
        u + (s + 1)(c - u).  The head is linear after the final RMSNorm, so the
        combination is taken on the normalised hidden rows, (s + 1) n_c - s n_u,
        and the vocabulary GEMM runs once over B rows instead of twice.
        """
        B, L = tokens.shape
        if guidance > 0 and B % 2:
            raise ValueError("guided logits need conditional and unconditional halves")
        h = self.hidden(tokens, layer_limit)
        if rows is not None:
            R = rows.shape[1]
            flat = (torch.arange(B, device=self.device)[:, None] * L + rows.to(self.device)).reshape(-1)
            sel = self._buf("sel", (B * R, self.cfg.hidden_size))
            torch.index_select(h, 0, flat, out=sel)
        else:
            R = L
            sel = h
        xn = self._buf("xn", sel.shape)
        K.rmsnorm(sel, self.w.final_norm, self.cfg.rms_norm_eps, out=xn)
        if guidance > 0:
            half = xn.shape[0] // 2
            xn = ((guidance + 1.0) * xn[:half].float() - guidance * xn[half:].float()).to(torch.bfloat16)
            B //= 2
        out = torch.empty(xn.shape[0], self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        K.linear(xn, self.w.head, out=out, out_dtype=torch.float32, static_weights=True)
        return out.view(B, R, -1)

    __call__ = logits


def reference_forward(config: MoEConfig, sd: dict[str, torch.Tensor], tokens: torch.Tensor) -> torch.Tensor:
    """Plain fp32 PyTorch forward (bidirectional) of one sequence: logits [L, V]."""
    f = {k: v.float() for k, v in sd.items()}
    D, eps = config.head_dim, config.rms_norm_eps
    nq, nkv = config.num_attention_heads, config.num_key_value_heads
    F = config.moe_intermediate_size

    def rms(x, w):
        return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w

    x = f["model.embed_tokens.weight"][tokens.long()]
    L = x.shape[0]
    inv = K.rope_frequencies(D, config.rope_theta)
    ang = torch.arange(L, dtype=torch.float32)[:, None] * inv[None]
    cos, sin = ang.cos(), ang.sin()

    def rope(t):
        a, b = t[..., : D // 2], t[..., D // 2:]
        return torch.cat((a * cos[:, None] - b * sin[:, None], b * cos[:, None] + a * sin[:, None]), -1)

    for i in range(config.num_hidden_layers):
        p = f"model.layers.{i}."
        hn = rms(x, f[p + "input_layernorm.weight"])
        q = (hn @ f[p + "self_attn.q_proj.weight"].t()).view(L, nq, D)
        k = (hn @ f[p + "self_attn.k_proj.weight"].t()).view(L, nkv, D)
        v = (hn @ f[p + "self_attn.v_proj.weight"].t()).view(L, nkv, D)
        if config.qk_norm:
            q, k = rms(q, f[p + "self_attn.q_norm.weight"]), rms(k, f[p + "self_attn.k_norm.weight"])
        q, k = rope(q), rope(k)
        G = nq // nkv
        k, v = k.repeat_interleave(G, 1), v.repeat_interleave(G, 1)
        s = torch.einsum("qhd,khd->hqk", q, k) / math.sqrt(D)
        o = torch.einsum("hqk,khd->qhd", s.softmax(-1), v).reshape(L, nq * D)
        x = x + o @ f[p + "self_attn.o_proj.weight"].t()
        hn = rms(x, f[p + "post_attention_layernorm.weight"])
        probs = (hn @ f[p + "mlp.gate.weight"].t()).softmax(-1)
        order = torch.sort(-probs, dim=-1, stable=True).indices[:, : config.num_experts_per_tok]
        wts = probs.gather(-1, order)
        if config.norm_topk_prob:
            wts = wts / wts.sum(-1, keepdim=True)
        moe = torch.zeros_like(x)
        for j in range(order.shape[1]):
            for e in order[:, j].unique().tolist():
                rows = (order[:, j] == e).nonzero(as_tuple=True)[0]
                g = hn[rows] @ f[p + f"mlp.experts.{e}.gate_proj.weight"].t()
                u = hn[rows] @ f[p + f"mlp.experts.{e}.up_proj.weight"].t()
                y = (torch.nn.functional.silu(g) * u) @ f[p + f"mlp.experts.{e}.down_proj.weight"].t()
                moe[rows] += wts[rows, j, None] * y
        x = x + moe
    x = rms(x, f["model.norm.weight"])
    head = f["model.embed_tokens.weight"] if config.tie_word_embeddings else f["lm_head.weight"]
    return x @ head.t()
