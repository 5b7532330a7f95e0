"""VRPO training of LoRA adapters on the LLaDA-MoE-shaped masked-diffusion model.

Reference behaviour: experiments/dllm/train_gsm8k_vrpo.py:221-450 (PEFT LoRA on
LLaDA-MoE, ``estimate_vrpo_preference_loss`` per pair, gradient accumulation,
AdamW, adapter + optimizer checkpoints with a fingerprinted resume) and the
``[vrpo_training]`` / ``[vrpo_lora]`` settings of
configs/gsm8k_llada_moe_3090.toml.

B200 design:
* the base weights stay frozen bf16 in kernel layout (``models.moe``); the
  policy's training forward uses the tcgen05 GEMM for every projection, the
  LoRA term is added through the GEMM residual epilogue, the MoE layer is the
  kernel forward with a grouped-GEMM backward (``training.moe_autograd``),
  attention is PyTorch SDPA (bidirectional);
* the ELBO only needs log-probabilities at masked positions: hidden states of
  those rows go through the fused chunked head + log-probability op, so no
  [rows x vocab] logits tensor exists;
* the reference policy is the same resident weights with the adapters off
  (``disable_adapter``), evaluated without autograd;
* all adapter tensors are views of one flat fp32 buffer: data-parallel ranks
  all-reduce one gradient buffer and the fused AdamW kernel updates it in one
  launch.
"""

from __future__ import annotations

import hashlib
import json
import math
import time
from contextlib import contextmanager
from dataclasses import asdict, dataclass, field
from pathlib import Path
from typing import Sequence

import torch
import torch.nn.functional as F

from ..dllm.config import VRPOSamplingConfig
from ..dllm.vrpo import AdapterDisabledReference, estimate_vrpo_preference_loss
from ..models.moe import MoEConfig, MoEWeights
from ..ops import kernels as K
from .lora import LoRAConfig, LoRAParameters, lora_linear
from .moe_autograd import FrozenExperts, moe_ffn_autograd, moe_ffn_lora

FORMAT = "vrpo-lora-v1"

# The reference's [vrpo_lora] target modules (configs/gsm8k_llada_moe_3090.toml): the
# attention projections and every expert's gate / up / down projection.
VRPO_TARGETS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
SUPPORTED_TARGETS = frozenset(VRPO_TARGETS)


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)).to(torch.bfloat16) * w


def _rope(t, cos, sin):
    half = t.shape[-1] // 2
    a, b = t[..., :half].float(), t[..., half:].float()
    return torch.cat((a * cos - b * sin, b * cos + a * sin), -1).to(torch.bfloat16)


class LoRAMoEPolicy:
    """Masked-diffusion policy = frozen MoE weights + LoRA adapters.

    Targets: the attention projections (q / k / v on the fused QKV weight with
    per-projection blocks, o) and every expert's gate / up (one block-masked
    adapter per expert on the interleaved gate / up rows) and down projection.
    The default is the reference's full target list (``VRPO_TARGETS``, r 16,
    alpha 32, dropout 0.05).
    """

    def __init__(self, weights: MoEWeights, lora: LoRAConfig = LoRAConfig(dropout=0.05, targets=VRPO_TARGETS), *,
                 seed: int = 0, head_chunk_rows: int = 2048):
        unknown = set(lora.targets) - SUPPORTED_TARGETS
        if unknown:
            raise ValueError(f"LoRA targets not supported on this model: {sorted(unknown)}")
        self.w = weights
        self.cfg: MoEConfig = weights.config
        self.lora = lora
        self.device = weights.embed.device
        self.training = True
        self._disabled = False
        self.head_chunk_rows = head_chunk_rows
        c = self.cfg
        D, nq, nkv, H = c.head_dim, c.num_attention_heads, c.num_key_value_heads, c.hidden_size
        gen = torch.Generator().manual_seed(seed)
        self.adapters: list[dict[str, LoRAParameters]] = []
        qkv_targets = [t for t in ("q_proj", "k_proj", "v_proj") if t in lora.targets]
        for _ in range(c.num_hidden_layers):
            layer = {}
            if qkv_targets:
                # fused QKV with per-projection adapters; projections without a target get a zero block (masked)
                layer["qkv"] = _qkv_adapter(H, nq, nkv, D, lora.rank, qkv_targets, self.device, gen)
            if "o_proj" in lora.targets:
                layer["o"] = LoRAParameters(nq * D, H, lora.rank, device=self.device, generator=gen)
            gu_targets = [t for t in ("gate_proj", "up_proj") if t in lora.targets]
            for e in range(c.num_experts):
                if gu_targets:
                    layer[f"gu{e}"] = _gate_up_adapter(H, c.moe_intermediate_size, lora.rank, gu_targets, self.device,
                                                       gen)
                if "down_proj" in lora.targets:
                    layer[f"down{e}"] = LoRAParameters(c.moe_intermediate_size, H, lora.rank, device=self.device,
                                                       generator=gen)
            self.adapters.append(layer)
        self._flatten()
        self.experts = [FrozenExperts(lw.router, lw.w_gu, lw.w_down, c.num_experts_per_tok, c.norm_topk_prob)
                        for lw in weights.layers]
        self.anchor = torch.zeros((), device=self.device, requires_grad=True)

    # ---- parameters ----
    def _flatten(self):
        params = [p for layer in self.adapters for a in layer.values() for p in a.parameters()]
        n = sum(p.numel() for p in params)
        self.flat = torch.zeros(n, dtype=torch.float32, device=self.device, requires_grad=True)
        off = 0
        views = []
        for layer in self.adapters:
            for a in layer.values():
                for name in ("A", "B"):
                    t = getattr(a, name)
                    with torch.no_grad():
                        self.flat.data[off:off + t.numel()].copy_(t.detach().reshape(-1))
                    v = self.flat[off:off + t.numel()].view(t.shape)
                    setattr(a, name, v)
                    views.append((a, name, off, t.shape))
                    off += t.numel()
        self._views = views
        self.trainable = n

    def _refresh_views(self):
        # views must be re-derived from the leaf after every backward (their graph nodes are per-forward)
        for a, name, off, shape in self._views:
            setattr(a, name, self.flat[off:off + math.prod(shape)].view(shape))

    def parameters(self):
        return [self.flat]

    def train(self, mode: bool = True):
        self.training = mode
        return self

    def eval(self):
        return self.train(False)

    @contextmanager
    def disable_adapter(self):
        prev = self._disabled
        self._disabled = True
        try:
            yield
        finally:
            self._disabled = prev

    @torch.no_grad()
    def merged_weights(self) -> MoEWeights:
        """Serving weights with the adapters folded in: W + scale * (B * mask) @ A (other tensors shared)."""
        import dataclasses

        self._refresh_views()
        s = self.lora.scale
        layers = []
        E, Fd, H = self.cfg.num_experts, self.cfg.moe_intermediate_size, self.cfg.hidden_size
        for lw, ad in zip(self.w.layers, self.adapters):
            upd = {}
            for key, name in (("qkv", "w_qkv"), ("o", "w_o")):
                a = ad.get(key)
                if a is not None:
                    w = getattr(lw, name)
                    delta = s * ((a.B * a.block_mask) @ a.A)
                    upd[name] = (w.float() + delta.to(w.device)).to(w.dtype).contiguous()
            for prefix, name, rows in (("gu", "w_gu", 2 * Fd), ("down", "w_down", H)):
                if f"{prefix}0" not in ad:
                    continue
                w = getattr(lw, name).float().clone()
                for e in range(E):
                    a = ad[f"{prefix}{e}"]
                    w[e * rows:(e + 1) * rows] += s * ((a.B * a.block_mask) @ a.A).to(w.device)
                upd[name] = w.to(getattr(lw, name).dtype).contiguous()
            layers.append(dataclasses.replace(lw, **upd))
        return dataclasses.replace(self.w, layers=layers)

    # ---- forward ----
    def hidden(self, tokens: torch.Tensor) -> torch.Tensor:
        c = self.cfg
        self._refresh_views()
        B, L = tokens.shape
        D, nq, nkv, eps = c.head_dim, c.num_attention_heads, c.num_key_value_heads, c.rms_norm_eps
        use = not self._disabled
        s = self.lora.scale
        drop = self.lora.dropout if self.training else 0.0
        h = self.w.embed[tokens.to(self.device)]
        ang = torch.arange(L, device=self.device, dtype=torch.float32)[:, None] * self.w.inv_freq[None]
        cos, sin = ang.cos()[None, :, None], ang.sin()[None, :, None]
        for lw, ad, ex in zip(self.w.layers, self.adapters, self.experts):
            x = _rms(h, lw.in_norm, eps).reshape(B * L, -1)
            qkv = lora_linear(x, lw.w_qkv, ad.get("qkv") if use else None, s, dropout=drop,
                              training=self.training).view(B, L, -1)
            q = qkv[..., : nq * D].reshape(B, L, nq, D)
            k = qkv[..., nq * D:(nq + nkv) * D].reshape(B, L, nkv, D)
            v = qkv[..., (nq + nkv) * D:].reshape(B, L, nkv, D)
            if lw.q_norm is not None:
                q, k = _rms(q, lw.q_norm, eps), _rms(k, lw.k_norm, eps)
            q, k = _rope(q, cos, sin), _rope(k, cos, sin)
            att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                 enable_gqa=nq != nkv)
            att = att.transpose(1, 2).reshape(B * L, nq * D)
            h = h + lora_linear(att, lw.w_o, ad.get("o") if use else None, s, dropout=drop,
                                training=self.training).view(B, L, -1)
            x = _rms(h, lw.post_norm, eps).reshape(B * L, -1)
            if "gu0" in ad or "down0" in ad:
                # with the adapters off (the reference policy) the same expert path runs without
                # the LoRA terms, so policy and reference agree bit for bit while B is zero
                E = self.cfg.num_experts
                h = moe_ffn_lora(x, h.reshape(B * L, -1), ex,
                                 [ad.get(f"gu{e}") if use else None for e in range(E)],
                                 [ad.get(f"down{e}") if use else None for e in range(E)], s, dropout=drop,
                                 training=self.training).view(B, L, -1)
            else:
                h = moe_ffn_autograd(x, h.reshape(B * L, -1), ex, self.anchor).view(B, L, -1)
        return h.reshape(B * L, -1)

    def masked_logprobs(self, tokens: torch.Tensor, flat_index: torch.Tensor, targets: torch.Tensor, *,
                        cfg_scale: float = 0.0, unconditional: torch.Tensor | None = None) -> torch.Tensor:
        """log p(target) at the given flattened (row * L + position) indices.

        With ``cfg_scale`` > 0 the logits are classifier-free guided,
        u + (s + 1)(c - u), where u comes from ``unconditional`` (the same rows
        with the prompt masked), as in the reference's ELBO.
        """
        idx = flat_index.to(self.device)
        h = self.hidden(tokens)
        sel = _rms(h[idx], self.w.final_norm, self.cfg.rms_norm_eps)
        if cfg_scale <= 0:
            return K.head_logprob(sel, self.w.head, targets.to(self.device), chunk_rows=self.head_chunk_rows)
        if unconditional is None:
            raise ValueError("classifier-free guidance needs the unconditional (prompt-masked) rows")
        hu = self.hidden(unconditional)
        sel_u = _rms(hu[idx], self.w.final_norm, self.cfg.rms_norm_eps)
        return _guided_logprob(sel, sel_u, self.w.head, targets.to(self.device), float(cfg_scale),
                               self.head_chunk_rows)


def _guided_chunk(c: torch.Tensor, u: torch.Tensor, head: torch.Tensor, t: torch.Tensor, s: float) -> torch.Tensor:
    lc = (c.to(torch.bfloat16) @ head.t()).float()
    lu = (u.to(torch.bfloat16) @ head.t()).float()
    return (lu + (s + 1.0) * (lc - lu)).log_softmax(-1).gather(1, t[:, None].long()).squeeze(1)


def _guided_logprob(c: torch.Tensor, u: torch.Tensor, head: torch.Tensor, targets: torch.Tensor, s: float,
                    chunk: int) -> torch.Tensor:
    """log softmax(u + (s + 1)(c - u))[target] per row, logits from hidden rows c / u and
    the head; row chunks are recomputed in the backward instead of keeping [rows, V]."""
    from torch.utils.checkpoint import checkpoint

    outs = []
    for i in range(0, c.shape[0], chunk):
        outs.append(checkpoint(_guided_chunk, c[i:i + chunk], u[i:i + chunk], head, targets[i:i + chunk], s,
                               use_reentrant=False))
    return torch.cat(outs)


def _gate_up_adapter(H, Fd, r, targets, device, gen) -> LoRAParameters:
    """One expert's gate / up adapter on the interleaved [64 gate | 64 up] rows of its
    fused weight: A stacks a gate and an up block [2r, H]; B [2F, 2r] is masked so
    gate rows read the gate block and up rows the up block (a projection that is not
    a target keeps all-zero rows)."""
    a = LoRAParameters(H, 2 * Fd, r, groups=1, device=device, generator=gen)
    a.A = torch.cat([((torch.rand(r, H, generator=gen) * 2 - 1) / math.sqrt(H)) for _ in range(2)]).to(
        device).requires_grad_(True)
    a.B = torch.zeros(2 * Fd, 2 * r, device=device, requires_grad=True)
    row = torch.arange(2 * Fd, device=device)
    is_up = (row % 128) >= 64
    mask = torch.zeros(2 * Fd, 2 * r, device=device)
    if "gate_proj" in targets:
        mask[~is_up, :r] = 1
    if "up_proj" in targets:
        mask[is_up, r:] = 1
    a.block_mask = mask
    a.groups = 2
    return a


def _qkv_adapter(H, nq, nkv, D, r, targets, device, gen) -> LoRAParameters:
    a = LoRAParameters(H, (nq + 2 * nkv) * D, r, groups=1, device=device, generator=gen)
    # per-projection blocks: A stacks three [r, H] blocks, B is block diagonal over (q | k | v)
    sizes = (nq * D, nkv * D, nkv * D)
    names = ("q_proj", "k_proj", "v_proj")
    a.A = torch.cat([((torch.rand(r, H, generator=gen) * 2 - 1) / math.sqrt(H)) for _ in names]).to(
        device).requires_grad_(True)
    a.B = torch.zeros(sum(sizes), 3 * r, device=device, requires_grad=True)
    mask = torch.zeros(sum(sizes), 3 * r, device=device)
    row = 0
    for g, (n, name) in enumerate(zip(sizes, names)):
        if name in targets:
            mask[row:row + n, g * r:(g + 1) * r] = 1
        row += n
    a.block_mask = mask
    a.groups = 3
    return a


@dataclass(frozen=True)
class VRPOTrainingConfig:
    learning_rate: float = 5e-6
    beta: float = 0.04
    gradient_accumulation_steps: int = 4
    max_grad_norm: float = 1.0
    weight_decay: float = 0.0
    sampling: VRPOSamplingConfig = field(default_factory=VRPOSamplingConfig)
    seed: int = 20260808

    def __post_init__(self):
        if self.learning_rate <= 0 or self.beta <= 0 or self.gradient_accumulation_steps < 1:
            raise ValueError("positive learning rate / beta and accumulation required")


class VRPOTrainer:
    def __init__(self, policy: LoRAMoEPolicy, pairs: Sequence[tuple[tuple[int, ...], tuple[int, ...], tuple[int, ...]]],
                 config: VRPOTrainingConfig = VRPOTrainingConfig(), *, group=None):
        if not pairs:
            raise ValueError("at least one preference pair is required")
        self.policy, self.pairs, self.config, self.group = policy, list(pairs), config, group
        self.reference = AdapterDisabledReference(policy)
        self.exp_avg = torch.zeros_like(policy.flat.data)
        self.exp_avg_sq = torch.zeros_like(policy.flat.data)
        self.step = 0
        self.cursor = 0
        self.world = 1
        if group is not None:
            import torch.distributed as dist

            self.world = dist.get_world_size(group)
        self.history: list[dict] = []

    def fingerprint(self) -> str:
        h = hashlib.sha256(json.dumps({"model": self.policy.cfg.to_dict(), "lora": asdict(self.policy.lora),
                                       "config": _jsonable(asdict(self.config))}, sort_keys=True).encode())
        return h.hexdigest()

    def train_step(self) -> dict:
        c = self.config
        t0 = time.perf_counter()
        p = self.policy
        if p.flat.grad is not None:
            p.flat.grad = None
        losses, scores = [], []
        mask_id = p.cfg.mask_token_id
        for _ in range(c.gradient_accumulation_steps):
            prompt, chosen, rejected = self.pairs[self.cursor % len(self.pairs)]
            est = estimate_vrpo_preference_loss(p, self.reference, prompt=prompt, chosen=chosen, rejected=rejected,
                                                mask_token_id=mask_id, config=c.sampling, beta=c.beta,
                                                seed=c.seed * 1000003 + self.cursor)
            (est.loss / c.gradient_accumulation_steps).backward()
            losses.append(float(est.loss.detach()))
            scores.append(float(est.preference_score.detach()))
            self.cursor += 1
        g = p.flat.grad if p.flat.grad is not None else torch.zeros_like(p.flat.data)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(g, group=self.group)
            g.div_(self.world)
        self.step += 1
        sq = K.adamw_step(p.flat.data, g.contiguous(), self.exp_avg, self.exp_avg_sq, step=self.step,
                          lr=c.learning_rate, weight_decay=c.weight_decay, clip=c.max_grad_norm)
        p.flat.grad = None
        rec = {"step": self.step, "loss": sum(losses) / len(losses), "preference_score": sum(scores) / len(scores),
               "grad_norm": float(sq.sqrt()) if sq is not None else None, "seconds": time.perf_counter() - t0}
        self.history.append(rec)
        return rec

    def save(self, path) -> None:
        torch.save({"format": FORMAT, "fingerprint": self.fingerprint(), "adapters": self.policy.flat.detach().cpu(),
                    "exp_avg": self.exp_avg.cpu(), "exp_avg_sq": self.exp_avg_sq.cpu(), "step": self.step,
                    "cursor": self.cursor, "lora": asdict(self.policy.lora), "history": self.history}, path)

    def resume(self, path) -> None:
        st = torch.load(path, weights_only=False)
        if st.get("format") != FORMAT:
            raise ValueError("not a VRPO adapter checkpoint")
        if st["fingerprint"] != self.fingerprint():
            raise ValueError("checkpoint fingerprint differs from this model / LoRA / training configuration")
        with torch.no_grad():
            self.policy.flat.copy_(st["adapters"].to(self.policy.device))
        self.exp_avg.copy_(st["exp_avg"].to(self.exp_avg.device))
        self.exp_avg_sq.copy_(st["exp_avg_sq"].to(self.exp_avg_sq.device))
        self.step, self.cursor, self.history = int(st["step"]), int(st["cursor"]), list(st["history"])


def _jsonable(x):
    if isinstance(x, dict):
        return {k: _jsonable(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return [_jsonable(v) for v in x]
    return x


__all__ = ["FORMAT", "LoRAMoEPolicy", "VRPO_TARGETS", "VRPOTrainer", "VRPOTrainingConfig"]
