"""Causal decoder with token-gated low-rank projections, and noise-input drafting on it.

One set of base weights serves both roles. A boolean ``adapter_mask`` over the
input tokens turns on a low-rank update ``(alpha / r) B A x`` in the selected
projections for the marked rows only; unmarked rows run the plain decoder.

Drafting (:class:`NoiseBranch`): the input block is the clean anchor followed
by ``K - 1`` uniform noise tokens, in one causal forward over the read-only
history. The anchor row is unadapted and causal, so its logits are the exact
next-token law: the round draws its first token (the *root*) from it and
commits it without verification. The adapted noise rows propose the next
``K - 1`` tokens, which the ordinary verifier then checks. Because history and
anchor never pass through an adapter, their keys and values do not depend on
the adapter, which makes the online update (:class:`LowRankLearner`) an exact
gradient of the drafted rows alone.

Training (:func:`paired_batch`) packs ``[clean, noisy]`` side by side with
shared position ids. Noisy row ``j`` in the block that starts at ``s`` sees the
clean keys ``<= s`` (history plus the block's clean anchor) and the noisy keys
``s < i <= j``: exactly the visibility of the drafting forward, so the offline
loss trains the rows that decoding uses. The teacher is the clean side's own
row ``j`` (detached).

Parameter names follow the Hugging Face Qwen2/Qwen3 layout
(``model.layers.N.self_attn.q_proj.weight`` ...), so a Qwen checkpoint's state
dict loads into :class:`LowRankDecoder` unchanged (:func:`from_hf`).

Reference behaviour: online-speculation/ablation/src/blockspec_ablation/
model.py, attention.py, distillation.py, parallel/branches.py
(CausalLowRankBranch), decoding.py, online.py, hf_execution.py.
"""

from __future__ import annotations

import json
import math
import time
from dataclasses import asdict, dataclass, field
from pathlib import Path

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .diffusion import UniformNoise
from .generation import DraftBatch
from .model import cache_length, trim_cache

PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
ATTENTION_BACKENDS = ("sdpa", "grouped")
LOSS_KINDS = ("l1", "tv", "forward_kl", "reverse_kl", "reverse_kl_l1")
FORMAT = "blockspec-lowrank-v1"


@dataclass(frozen=True)
class LowRankConfig:
    vocab_size: int = 32
    hidden_size: int = 64
    intermediate_size: int = 128
    num_hidden_layers: int = 2
    num_attention_heads: int = 4
    num_key_value_heads: int = 2
    head_dim: int = 16
    rms_norm_eps: float = 1e-6
    norm_groups: int = 1
    query_key_norm: bool = False
    attention_bias: bool = False
    tie_word_embeddings: bool = False
    rope_theta: float = 10000.0
    rope_factor: float = 1.0              # YaRN extension factor; 1 is plain RoPE
    rope_original_length: int = 8192
    rope_beta_fast: float = 32.0
    rope_beta_slow: float = 1.0
    rope_attention_factor: float = 1.0
    adapter_rank: int = 8
    adapter_alpha: float = 8.0
    adapter_targets: tuple = PROJECTIONS

    def __post_init__(self):
        for name in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
                     "num_attention_heads", "num_key_value_heads", "head_dim", "norm_groups"):
            if getattr(self, name) < 1:
                raise ValueError(f"{name} must be positive")
        if self.head_dim % 2 or self.num_attention_heads % self.num_key_value_heads:
            raise ValueError("an even head dimension and whole query groups per KV head are required")
        if self.hidden_size % self.norm_groups or self.adapter_rank < 0:
            raise ValueError("invalid norm groups or adapter rank")
        targets = tuple(self.adapter_targets)
        if not set(targets) <= set(PROJECTIONS) or len(set(targets)) != len(targets):
            raise ValueError("adapter targets must be distinct projection names")
        object.__setattr__(self, "adapter_targets", targets)
        if not (self.rope_theta > 1 and self.rope_factor >= 1 and self.rope_beta_fast > self.rope_beta_slow > 0
                and self.rms_norm_eps > 0 and self.adapter_alpha > 0 and self.rope_attention_factor > 0):
            raise ValueError("invalid rotary, normalisation or adapter scale")

    def to_dict(self) -> dict:
        d = asdict(self)
        d["adapter_targets"] = list(self.adapter_targets)
        return d

    @classmethod
    def from_dict(cls, d: dict) -> "LowRankConfig":
        d = dict(d)
        if "adapter_targets" in d:
            d["adapter_targets"] = tuple(d["adapter_targets"])
        return cls(**d)

    @classmethod
    def from_hf(cls, hf: dict, **adapter) -> "LowRankConfig":
        """From a Qwen2 / Qwen3 / Llama ``config.json`` dictionary (YaRN ``rope_scaling`` included)."""
        heads = hf["num_attention_heads"]
        scaling = hf.get("rope_scaling") or {}
        yarn = scaling.get("rope_type", scaling.get("type")) == "yarn"
        factor = float(scaling.get("factor", 1.0)) if yarn else 1.0
        return cls(vocab_size=hf["vocab_size"], hidden_size=hf["hidden_size"],
                   intermediate_size=hf["intermediate_size"], num_hidden_layers=hf["num_hidden_layers"],
                   num_attention_heads=heads, num_key_value_heads=hf.get("num_key_value_heads", heads),
                   head_dim=hf.get("head_dim") or hf["hidden_size"] // heads,
                   rms_norm_eps=hf.get("rms_norm_eps", 1e-6),
                   query_key_norm=hf.get("model_type") == "qwen3",
                   attention_bias=bool(hf.get("attention_bias", hf.get("model_type") == "qwen2")),
                   tie_word_embeddings=bool(hf.get("tie_word_embeddings", False)),
                   rope_theta=float(hf.get("rope_theta", 10000.0)), rope_factor=factor,
                   rope_original_length=int(scaling.get("original_max_position_embeddings", 8192)),
                   rope_beta_fast=float(scaling.get("beta_fast", 32.0)),
                   rope_beta_slow=float(scaling.get("beta_slow", 1.0)),
                   rope_attention_factor=(float(scaling.get("attention_factor", 0.1 * math.log(factor) + 1.0))
                                          if yarn else 1.0), **adapter)


class GatedLinear(nn.Module):
    """``W x + b`` plus ``(alpha / r) B A x`` on the rows where ``mask`` is set; no mask, no adapter."""

    def __init__(self, inputs: int, outputs: int, rank: int, alpha: float, bias: bool = False):
        super().__init__()
        self.weight = nn.Parameter(torch.randn(outputs, inputs) * 0.02)
        self.bias = nn.Parameter(torch.zeros(outputs)) if bias else None
        self.rank, self.scale = rank, (alpha / rank if rank else 0.0)
        if rank:
            self.lora_A = nn.Parameter(torch.randn(rank, inputs) / math.sqrt(inputs))
            self.lora_B = nn.Parameter(torch.zeros(outputs, rank))   # a fresh adapter changes nothing

    def forward(self, x: Tensor, mask: Tensor | None = None) -> Tensor:
        out = F.linear(x, self.weight, self.bias)
        if not self.rank or mask is None:
            return out
        # the row gate commutes with B: gate in rank space, where the tensor is smallest
        low = F.linear(x, self.lora_A.to(x.dtype)) * mask[..., None].to(x.dtype)
        return out + F.linear(low, self.lora_B.to(x.dtype)) * self.scale


class GroupedRMSNorm(nn.Module):
    """RMS normalisation over ``groups`` equal slices of the last dimension (fp32 statistics)."""

    def __init__(self, width: int, eps: float, groups: int = 1):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))
        self.eps, self.groups = eps, groups

    def forward(self, x: Tensor) -> Tensor:
        w = x.float().reshape(*x.shape[:-1], self.groups, -1)
        w = w * torch.rsqrt(w.square().mean(-1, keepdim=True) + self.eps)
        return w.reshape_as(x).to(x.dtype) * self.weight


def rotary_frequencies(c: LowRankConfig, device=None) -> Tensor:
    """Inverse wavelengths of RoPE; with ``rope_factor > 1`` the NTK-by-parts ramp of YaRN
    (Peng et al., 2023): dimensions that turn more than ``beta_fast`` times over the original
    context keep their frequency, those under ``beta_slow`` turns are divided by the factor,
    and a linear ramp blends the dimensions between."""
    d = c.head_dim
    i = torch.arange(d // 2, dtype=torch.float32, device=device)
    inv = c.rope_theta ** (-2.0 * i / d)
    if c.rope_factor == 1:
        return inv

    def dim_for(turns):   # the dimension index whose wavelength fits ``turns`` times in the context
        return d * math.log(c.rope_original_length / (2 * math.pi * turns)) / (2 * math.log(c.rope_theta))

    lo = max(0, math.floor(dim_for(c.rope_beta_fast)))
    hi = min(d // 2 - 1, math.ceil(dim_for(c.rope_beta_slow)))
    ramp = ((i - lo) / max(hi - lo, 1e-3)).clamp(0, 1)
    return inv * (1 - ramp) + inv / c.rope_factor * ramp


def _rotate(x: Tensor, cos: Tensor, sin: Tensor) -> Tensor:
    h = x.shape[-1] // 2
    return x * cos + torch.cat((-x[..., h:], x[..., :h]), -1) * sin


def grouped_attention(q: Tensor, k: Tensor, v: Tensor, allowed: Tensor) -> Tensor:
    """Explicit masked softmax for short query blocks: the query heads of each KV group are
    stacked as rows against the shared K/V (no K/V repetition). ``q`` [B, H, T, D], ``k``/``v``
    [B, Hkv, S, D], ``allowed`` bool broadcastable to [B, H, T, S]. A row with no visible key
    returns zeros."""
    B, H, T, D = q.shape
    G = k.shape[1]
    s = (q.reshape(B, G, (H // G) * T, D) @ k.transpose(-1, -2)).reshape(B, H, T, -1) / math.sqrt(D)
    allowed = allowed.expand(B, H, T, s.shape[-1])
    if s.dtype in (torch.float16, torch.bfloat16):
        s = s.float()
    s = s.masked_fill(~allowed, float("-inf"))
    any_key = allowed.any(-1, keepdim=True)
    p = torch.where(any_key, s, 0.0).softmax(-1).masked_fill(~allowed, 0.0).to(v.dtype)
    return (p.reshape(B, G, (H // G) * T, -1) @ v).reshape(B, H, T, v.shape[-1])


class Attention(nn.Module):
    def __init__(self, c: LowRankConfig):
        super().__init__()
        self.config, self.backend = c, "sdpa"

        def proj(name, i, o, bias):
            return GatedLinear(i, o, c.adapter_rank if name in c.adapter_targets else 0, c.adapter_alpha, bias)

        self.q_proj = proj("q_proj", c.hidden_size, c.num_attention_heads * c.head_dim, c.attention_bias)
        self.k_proj = proj("k_proj", c.hidden_size, c.num_key_value_heads * c.head_dim, c.attention_bias)
        self.v_proj = proj("v_proj", c.hidden_size, c.num_key_value_heads * c.head_dim, c.attention_bias)
        self.o_proj = proj("o_proj", c.num_attention_heads * c.head_dim, c.hidden_size, False)
        if c.query_key_norm:
            self.q_norm = GroupedRMSNorm(c.head_dim, c.rms_norm_eps)
            self.k_norm = GroupedRMSNorm(c.head_dim, c.rms_norm_eps)

    def forward(self, x, mask, past, rotary, allowed):
        c, (B, T, _) = self.config, x.shape
        q = self.q_proj(x, mask).view(B, T, c.num_attention_heads, c.head_dim)
        k = self.k_proj(x, mask).view(B, T, c.num_key_value_heads, c.head_dim)
        v = self.v_proj(x, mask).view(B, T, c.num_key_value_heads, c.head_dim).transpose(1, 2)
        if c.query_key_norm:
            q, k = self.q_norm(q), self.k_norm(k)
        cos, sin = rotary
        q, k = _rotate(q.transpose(1, 2), cos, sin), _rotate(k.transpose(1, 2), cos, sin)
        if isinstance(past, WorkspaceLayer):
            k, v = past.write(k, v)
        elif past is not None:
            k, v = torch.cat((past[0], k), 2), torch.cat((past[1], v), 2)
        if self.backend == "grouped":
            o = grouped_attention(q, k, v, allowed)
        else:
            o = F.scaled_dot_product_attention(q, k, v, attn_mask=allowed, enable_gqa=True)
        return self.o_proj(o.transpose(1, 2).reshape(B, T, -1), mask), (k, v)


class MLP(nn.Module):
    def __init__(self, c: LowRankConfig):
        super().__init__()

        def proj(name, i, o):
            return GatedLinear(i, o, c.adapter_rank if name in c.adapter_targets else 0, c.adapter_alpha)

        self.gate_proj = proj("gate_proj", c.hidden_size, c.intermediate_size)
        self.up_proj = proj("up_proj", c.hidden_size, c.intermediate_size)
        self.down_proj = proj("down_proj", c.intermediate_size, c.hidden_size)

    def forward(self, x, mask):
        return self.down_proj(F.silu(self.gate_proj(x, mask)) * self.up_proj(x, mask), mask)


class Layer(nn.Module):
    def __init__(self, c: LowRankConfig):
        super().__init__()
        self.input_layernorm = GroupedRMSNorm(c.hidden_size, c.rms_norm_eps, c.norm_groups)
        self.post_attention_layernorm = GroupedRMSNorm(c.hidden_size, c.rms_norm_eps, c.norm_groups)
        self.self_attn = Attention(c)
        self.mlp = MLP(c)

    def forward(self, x, mask, past, rotary, allowed):
        a, kv = self.self_attn(self.input_layernorm(x), mask, past, rotary, allowed)
        x = x + a
        return x + self.mlp(self.post_attention_layernorm(x), mask), kv


class Body(nn.Module):
    def __init__(self, c: LowRankConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(c.vocab_size, c.hidden_size)
        nn.init.normal_(self.embed_tokens.weight, std=0.02)
        self.layers = nn.ModuleList(Layer(c) for _ in range(c.num_hidden_layers))
        self.norm = GroupedRMSNorm(c.hidden_size, c.rms_norm_eps, c.norm_groups)


@dataclass
class WorkspaceLayer:
    """One layer of a fixed-capacity KV workspace: this forward's rows are written in place at
    ``index`` (their positions) and attention reads the whole capacity under the caller's mask."""

    k: Tensor          # [1, Hkv, capacity, D]
    v: Tensor
    index: Tensor      # [T] write positions

    def write(self, k: Tensor, v: Tensor):
        self.k.index_copy_(2, self.index, k.to(self.k.dtype))
        self.v.index_copy_(2, self.index, v.to(self.v.dtype))
        return self.k, self.v


@dataclass
class Boundary:
    """The residual stream entering layer ``start`` of one forward, enough to recompute the suffix."""

    hidden: Tensor
    positions: Tensor
    allowed: Tensor
    adapter_mask: Tensor | None
    start: int


@dataclass
class LowRankOutput:
    logits: Tensor
    cache: tuple | None = None
    boundary: Boundary | None = None


def is_adapter(name: str) -> bool:
    return name.endswith((".lora_A", ".lora_B"))


class LowRankDecoder(nn.Module):
    def __init__(self, config: LowRankConfig = LowRankConfig()):
        super().__init__()
        self.config = config
        self.model = Body(config)
        self.lm_head = nn.Linear(config.hidden_size, config.vocab_size, bias=False)
        nn.init.normal_(self.lm_head.weight, std=0.02)
        if config.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        self.register_buffer("frequencies", rotary_frequencies(config), persistent=False)

    def _apply(self, fn, recurse=True):
        super()._apply(fn, recurse=recurse)
        # a dtype cast of the module keeps the rotary table in fp32
        self.frequencies = rotary_frequencies(self.config, device=self.lm_head.weight.device)
        return self

    def set_attention_backend(self, backend: str) -> "LowRankDecoder":
        if backend not in ATTENTION_BACKENDS:
            raise ValueError(f"attention backend must be one of {ATTENTION_BACKENDS}")
        for layer in self.model.layers:
            layer.self_attn.backend = backend
        return self

    def set_base_dtype(self, dtype) -> "LowRankDecoder":
        """Cast the base weights (bf16 execution); adapters keep their stored precision."""
        if dtype not in (torch.float32, torch.bfloat16):
            raise ValueError("base weights run in fp32 or bf16")
        for n, p in self.named_parameters():
            if not is_adapter(n):
                p.data = p.data.to(dtype)
        return self

    def adapter_parameters(self) -> list:
        return [p for n, p in self.named_parameters() if is_adapter(n)]

    def train_adapters_only(self) -> "LowRankDecoder":
        """Freeze the base; adapters train in fp32 whatever the base dtype."""
        for n, p in self.named_parameters():
            p.grad = None
            p.requires_grad_(is_adapter(n))
            if is_adapter(n):
                p.data = p.data.float()
        return self

    def _rotary(self, positions: Tensor, dtype):
        ang = positions.float()[..., None] * self.frequencies
        ang = torch.cat((ang, ang), -1)[:, None]
        f = self.config.rope_attention_factor
        return (ang.cos() * f).to(dtype), (ang.sin() * f).to(dtype)

    def _head(self, hidden: Tensor, logit_range):
        if logit_range is not None:
            a, b = logit_range
            if not 0 <= a < b <= hidden.shape[1]:
                raise ValueError("logit range must be a nonempty interval of the input")
            hidden = hidden[:, a:b]
        return self.lm_head(self.model.norm(hidden))

    def forward(self, tokens: Tensor, *, positions=None, allowed=None, adapter_mask=None, cache=None,
                capture_layer: int | None = None, logit_range=None) -> LowRankOutput:
        if tokens.ndim != 2 or tokens.shape[1] < 1:
            raise ValueError("tokens must be [batch, nonempty sequence]")
        B, T = tokens.shape
        past = cache_length(cache)
        if cache is not None and len(cache) != self.config.num_hidden_layers:
            raise ValueError("the cache has a different layer count")
        if positions is None:
            positions = torch.arange(past, past + T, device=tokens.device)[None].expand(B, -1)
        if positions.shape != tokens.shape or (adapter_mask is not None and adapter_mask.shape != tokens.shape):
            raise ValueError("positions and the adapter mask must match the tokens")
        if allowed is None:
            allowed = (torch.arange(past + T, device=tokens.device)[None]
                       <= past + torch.arange(T, device=tokens.device)[:, None])[None, None]
        if allowed.dtype != torch.bool or tuple(allowed.shape[-2:]) != (T, past + T):
            raise ValueError("allowed must be a boolean [.., queries, keys] mask")
        if capture_layer is not None and not 0 <= capture_layer <= self.config.num_hidden_layers:
            raise ValueError("capture layer out of range")
        h = self.model.embed_tokens(tokens)
        rotary = self._rotary(positions, h.dtype)
        new, boundary = [], None
        for i, layer in enumerate(self.model.layers):
            if i == capture_layer:
                boundary = Boundary(h, positions, allowed, adapter_mask, i)
            h, kv = layer(h, adapter_mask, None if cache is None else cache[i], rotary, allowed)
            new.append(kv)
        if capture_layer == self.config.num_hidden_layers:
            boundary = Boundary(h, positions, allowed, adapter_mask, capture_layer)
        return LowRankOutput(self._head(h, logit_range), tuple(new), boundary)

    def forward_workspace(self, tokens: Tensor, positions: Tensor, allowed: Tensor, adapter_mask, layers,
                          logit_range=None) -> Tensor:
        """Forward over a KV workspace (one :class:`WorkspaceLayer` per layer); fixed shapes, no
        host synchronisation, so it can be captured in a CUDA graph."""
        h = self.model.embed_tokens(tokens)
        rotary = self._rotary(positions, h.dtype)
        for layer, past in zip(self.model.layers, layers):
            h, _ = layer(h, adapter_mask, past, rotary, allowed)
        return self._head(h, logit_range)

    def forward_suffix(self, boundary: Boundary, *, cache=None, logit_range=None) -> Tensor:
        """Recompute layers ``boundary.start..`` from a captured boundary; ``cache`` holds those
        layers' history only."""
        n = self.config.num_hidden_layers - boundary.start
        if cache is not None and len(cache) != n:
            raise ValueError("the cache must cover exactly the suffix layers")
        h = boundary.hidden
        rotary = self._rotary(boundary.positions, h.dtype)
        for j in range(n):
            h, _ = self.model.layers[boundary.start + j](h, boundary.adapter_mask,
                                                         None if cache is None else cache[j], rotary,
                                                         boundary.allowed)
        return self._head(h, logit_range)


# --- weights -----------------------------------------------------------------------------------

def save(model: LowRankDecoder, path) -> None:
    torch.save({"format": FORMAT, "config": model.config.to_dict(),
                "state": {k: v.detach().cpu() for k, v in model.state_dict().items()}}, path)


def load(path, device="cpu") -> LowRankDecoder:
    blob = torch.load(path, map_location="cpu", weights_only=True)
    if blob.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    m = LowRankDecoder(LowRankConfig.from_dict(blob["config"]))
    m.load_state_dict(blob["state"])
    return m.to(device)


def from_hf(source, *, device="cpu", dtype=torch.bfloat16, **adapter) -> LowRankDecoder:
    """A frozen Hugging Face backbone (a ``transformers`` causal-LM module, or a directory with
    ``config.json`` and ``*.safetensors``) with fresh adapters. Parameter names are the HF ones, so
    the state dict maps one to one; only the adapter tensors are new."""
    if isinstance(source, nn.Module):
        cfg = LowRankConfig.from_hf(source.config.to_dict(), **adapter)
        state = source.state_dict()
    else:
        from safetensors.torch import load_file

        d = Path(source)
        cfg = LowRankConfig.from_hf(json.loads((d / "config.json").read_text()), **adapter)
        state = {}
        for f in sorted(d.glob("*.safetensors")):
            state.update(load_file(str(f)))
    m = LowRankDecoder(cfg)
    missing, unexpected = m.load_state_dict(state, strict=False)
    missing = [k for k in missing if not is_adapter(k) and not (cfg.tie_word_embeddings and k == "lm_head.weight")]
    unexpected = [k for k in unexpected if not k.endswith("rotary_emb.inv_freq")]
    if missing or unexpected:
        raise ValueError(f"checkpoint mismatch: missing {missing[:4]}, unexpected {unexpected[:4]}")
    return m.to(device).set_base_dtype(dtype).eval().requires_grad_(False)


_PEFT_PREFIX = "base_model.model."


def save_peft(model: LowRankDecoder, directory) -> None:
    """Write the adapters as a PEFT LoRA artifact (``adapter_config.json`` and
    ``adapter_model.safetensors`` with ``base_model.model.<module>.lora_A.weight`` keys)."""
    from safetensors.torch import save_file

    c, d = model.config, Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    (d / "adapter_config.json").write_text(json.dumps({
        "peft_type": "LORA", "task_type": "CAUSAL_LM", "r": c.adapter_rank, "lora_alpha": c.adapter_alpha,
        "target_modules": list(c.adapter_targets), "bias": "none", "lora_dropout": 0.0,
        "fan_in_fan_out": False, "use_rslora": False, "use_dora": False}, indent=1))
    save_file({f"{_PEFT_PREFIX}{n}.weight": p.detach().float().contiguous().cpu()
               for n, p in model.named_parameters() if is_adapter(n)}, str(d / "adapter_model.safetensors"))


def load_peft(model: LowRankDecoder, directory) -> dict:
    """Load a PEFT LoRA artifact into the adapters after checking all of it: plain LoRA (no DoRA,
    rsLoRA, bias, per-module rank or alpha), the model's rank, alpha and targets, and exactly
    the model's adapter tensors with their shapes. Nothing changes when a check fails."""
    from safetensors.torch import load_file

    d, c = Path(directory), model.config
    cfg = json.loads((d / "adapter_config.json").read_text())
    if (cfg.get("peft_type") != "LORA" or cfg.get("bias", "none") != "none" or cfg.get("use_dora")
            or cfg.get("use_rslora") or cfg.get("fan_in_fan_out") or cfg.get("rank_pattern")
            or cfg.get("alpha_pattern") or cfg.get("modules_to_save")):
        raise ValueError("only uniform, alpha / r scaled, bias-free LoRA adapters are supported")
    if (cfg.get("r") != c.adapter_rank or cfg.get("lora_alpha") != c.adapter_alpha
            or set(cfg.get("target_modules") or ()) != set(c.adapter_targets)):
        raise ValueError("the adapter's rank, alpha or targets differ from the model's")
    own = {n: p for n, p in model.named_parameters() if is_adapter(n)}
    state = {}
    for key, value in load_file(str(d / "adapter_model.safetensors")).items():
        if not key.startswith(_PEFT_PREFIX) or not key.endswith((".lora_A.weight", ".lora_B.weight")):
            raise ValueError(f"unexpected tensor {key}")
        state[key[len(_PEFT_PREFIX):-len(".weight")]] = value
    if set(state) != set(own) or any(state[n].shape != own[n].shape for n in own):
        raise ValueError("the adapter tensors do not match the model")
    with torch.no_grad():
        for n, p in own.items():
            p.copy_(state[n])
    return {"tensors": len(state), "rank": c.adapter_rank, "alpha": c.adapter_alpha}

# --- offline distillation ----------------------------------------------------------------------

@dataclass
class PairedBatch:
    tokens: Tensor         # [B, 2L]: clean then noisy
    positions: Tensor      # [B, 2L]: both halves share positions 0..L-1
    allowed: Tensor        # [1, 1, 2L, 2L]
    adapter_mask: Tensor   # [B, 2L]: the noisy non-anchor rows
    eligible: Tensor       # [B, L]: noisy rows with a teacher


def paired_batch(clean: Tensor, block_size: int, noisy: Tensor) -> PairedBatch:
    """Clean and noisy copies in one forward, with the drafting forward's visibility for every
    noisy row (module docstring). Positions ``j % block_size == 0`` are block anchors: clean,
    unadapted, never supervised."""
    if clean.ndim != 2 or clean.shape[1] < 2 or block_size < 2 or noisy.shape != clean.shape:
        raise ValueError("[batch, length >= 2] clean and noisy tokens and block_size >= 2 are required")
    B, L = clean.shape
    j = torch.arange(L, device=clean.device)
    start = (j // block_size) * block_size
    causal = j[None, :] <= j[:, None]
    allowed = torch.zeros(2 * L, 2 * L, dtype=torch.bool, device=clean.device)
    allowed[:L, :L] = causal
    allowed[L:, :L] = j[None, :] <= start[:, None]                        # clean history + anchor
    allowed[L:, L:] = causal & (j[None, :] > start[:, None])               # own block's noise so far
    drafted = (j % block_size != 0)[None].expand(B, -1)
    mask = torch.cat((torch.zeros_like(drafted), drafted), 1)
    return PairedBatch(torch.cat((clean, noisy), 1), j.repeat(2)[None].expand(B, -1), allowed[None, None],
                       mask, drafted)


def divergence(student: Tensor, teacher: Tensor, kind: str = "l1") -> Tensor:
    """Per-row divergence at temperature one. ``l1`` is the unhalved L1 distance (twice TV);
    ``reverse_kl`` is KL(student || teacher), ``forward_kl`` KL(teacher || student);
    ``reverse_kl_l1`` is their sum used as a warm-up."""
    if student.shape != teacher.shape:
        raise ValueError("student and teacher logits differ in shape")
    dt = torch.float64 if student.dtype == torch.float64 else torch.float32
    lq, lp = student.to(dt).log_softmax(-1), teacher.detach().to(dt).log_softmax(-1)
    q, p = lq.exp(), lp.exp()
    if kind in ("l1", "tv"):
        return (q - p).abs().sum(-1) * (0.5 if kind == "tv" else 1.0)
    if kind == "forward_kl":
        return (p * (lp - lq)).sum(-1)
    if kind == "reverse_kl":
        return (q * (lq - lp)).sum(-1)
    if kind == "reverse_kl_l1":
        return (q * (lq - lp)).sum(-1) + (q - p).abs().sum(-1)
    raise ValueError(f"loss kind must be one of {LOSS_KINDS}")


def paired_loss(model: LowRankDecoder, clean: Tensor, block_size: int, *, kind="l1", noise=UniformNoise(),
                generator=None) -> Tensor:
    noisy = noise.sample(clean.shape, model.config.vocab_size, device=clean.device, generator=generator)
    b = paired_batch(clean, block_size, noisy)
    logits = model(b.tokens, positions=b.positions, allowed=b.allowed, adapter_mask=b.adapter_mask).logits
    L = clean.shape[1]
    return divergence(logits[:, L:], logits[:, :L].detach(), kind)[b.eligible].mean()


def offline_step(model: LowRankDecoder, optimizer, clean: Tensor, block_size: int, *, kind="l1",
                 noise=UniformNoise(), generator=None, clip_norm: float = 1.0) -> dict:
    optimizer.zero_grad(set_to_none=True)
    loss = paired_loss(model, clean, block_size, kind=kind, noise=noise, generator=generator)
    if not torch.isfinite(loss):
        raise FloatingPointError("non-finite distillation loss")
    loss.backward()
    norm = torch.nn.utils.clip_grad_norm_(model.adapter_parameters(), clip_norm, error_if_nonfinite=True)
    optimizer.step()
    return {"loss": float(loss.detach()), "gradient_norm": float(norm)}


# --- drafting ----------------------------------------------------------------------------------

@dataclass
class NoiseDraft:
    """What a learner needs to recompute one drafting forward with gradients."""

    history: tuple | None
    inputs: Tensor
    route: Tensor


class NoiseBranch:
    """Generation branch for :func:`generation.generate` / :func:`generation.generate_ar`: the
    round's first token is the exact root from the clean anchor row, the noise rows propose the
    rest (module docstring)."""

    input_budget_extra = 0

    def __init__(self, model: LowRankDecoder, noise: UniformNoise = UniformNoise(), block_size: int = 8):
        self.model, self.noise, self.default_block_size = model, noise, block_size

    def ar(self, tokens: Tensor, cache=None, logits_to_keep: int = 0):
        out = self.model(tokens, cache=cache)
        return (out.logits[:, -logits_to_keep:] if logits_to_keep else out.logits), out.cache

    def draft(self, anchor: Tensor, cache, block_size: int, sampler, generator=None, feedback=None):
        noisy = self.noise.sample((1, block_size - 1), self.model.config.vocab_size, device=anchor.device,
                                  generator=generator)
        inputs = torch.cat((anchor, noisy), 1)
        route = torch.ones_like(inputs, dtype=torch.bool)
        route[:, 0] = False
        out = self.model(inputs, cache=cache, adapter_mask=route)
        root = sampler.sample_ar(out.logits[0, 0], generator)
        cand, q = sampler.propose(out.logits[0, 1:], generator)
        rooted = anchor.new_tensor([[root]])
        collect = feedback is not None and getattr(feedback, "learner", None) is not None
        return DraftBatch(torch.cat((rooted, cand[None]), 1), cand, q,
                          trim_cache(out.cache, cache_length(cache) + 1), [root], inputs,
                          NoiseDraft(cache, inputs, route) if collect else None, collect)


# --- online adapter learning -------------------------------------------------------------------

@dataclass
class _Observed:
    draft: NoiseDraft
    teacher: Tensor        # verifier logits for the supervised rows
    rows: int


@dataclass
class LowRankLearner:
    """Online adapter updates from verified rounds. Draft row ``i`` (noise input) proposed the
    token that the verifier's row ``i - 1`` scores, so the first ``used`` verifier rows are the
    teachers of draft rows ``1..used``; the loss recomputes only the drafting forward."""

    model: LowRankDecoder
    learning_rate: float = 1e-4
    interval: int = 1
    kind: str = "tv"
    clip_norm: float = 1.0
    updates: int = 0
    feedback_blocks: int = 0
    update_seconds: float = 0.0
    last_loss: float | None = None
    _pending: list = field(default_factory=list)

    def __post_init__(self):
        if self.interval < 1 or self.kind not in LOSS_KINDS:
            raise ValueError("a positive interval and a known loss kind are required")
        self.model.train_adapters_only()
        self.optimizer = torch.optim.Adam(self.model.adapter_parameters(), lr=self.learning_rate)

    def loss(self, items) -> Tensor:
        total, rows = 0.0, 0
        for it in items:
            out = self.model(it.draft.inputs, cache=it.draft.history, adapter_mask=it.draft.route,
                             logit_range=(1, 1 + it.rows))
            total = total + divergence(out.logits[0], it.teacher, self.kind).sum()
            rows += it.rows
        return total / rows

    def observe(self, draft: NoiseDraft, teacher_logits: Tensor, used: int, *, may_update: bool = True):
        rows = min(used, draft.inputs.shape[1] - 1)
        if rows < 1:
            return
        self._pending.append(_Observed(draft, teacher_logits[:rows].detach(), rows))
        self.feedback_blocks += 1
        if may_update and len(self._pending) >= self.interval:
            self.step()

    def step(self):
        if not self._pending:
            return
        t0 = time.perf_counter()
        with torch.enable_grad():
            self.optimizer.zero_grad(set_to_none=True)
            loss = self.loss(self._pending)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(self.model.adapter_parameters(), self.clip_norm)
            self.optimizer.step()
        self._pending.clear()
        self.updates += 1
        self.last_loss = float(loss.detach())
        self.update_seconds += time.perf_counter() - t0


class LowRankFeedback:
    """Generation hooks that feed verified rounds of a :class:`NoiseBranch` to a learner."""

    capture_layer = None

    def __init__(self, learner: LowRankLearner):
        self.learner = learner

    def begin(self, prompt):
        self._start = (self.learner.updates, self.learner.update_seconds, self.learner.feedback_blocks)
        self.learner._pending.clear()

    def commit(self, tokens):
        pass

    def observe(self, proposal, teacher_logits, target, *, used, fully_covered, done):
        if proposal.collect_feedback and proposal.boundary is not None:
            self.learner.observe(proposal.boundary, teacher_logits, used, may_update=not done)

    def finish(self, result):
        self.learner._pending.clear()
        u, s, f = self._start
        result.updates = self.learner.updates - u
        result.update_seconds = self.learner.update_seconds - s
        result.feedback_blocks = self.learner.feedback_blocks - f


__all__ = ["LowRankConfig", "GatedLinear", "WorkspaceLayer", "GroupedRMSNorm", "LowRankDecoder", "LowRankOutput", "Boundary",
           "grouped_attention", "rotary_frequencies", "is_adapter", "save", "load", "from_hf", "save_peft", "load_peft", "PairedBatch",
           "paired_batch", "divergence", "paired_loss", "offline_step", "NoiseBranch", "NoiseDraft",
           "LowRankLearner", "LowRankFeedback", "ATTENTION_BACKENDS", "LOSS_KINDS", "PROJECTIONS"]
