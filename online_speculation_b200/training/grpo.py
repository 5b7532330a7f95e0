"""GRPO training of a Qwen2 / Qwen3-shaped decoder on the sm_100a kernels, data parallel.

One step on every rank: sample ``group_size`` completions for each of
``prompts_per_rank`` prompts with the current policy (EngineBackend: paged KV,
graphed decode, on the very bf16 weights the trainer updates), score rewards,
form group-normalised advantages, compute per-token log-probabilities of the
frozen reference copy, then minimise the GRPO objective

    ratio_t = exp(logp_t - logp_old_t)            (logp_old = logp.detach())
    kl_t    = exp(ref_t - logp_t) - (ref_t - logp_t) - 1
    loss    = -mean_seq( sum_t m_t [min(ratio_t A, clip(ratio_t, 1-eps, 1+eps) A) - beta kl_t] / sum_t m_t )

with ``m`` the completion mask (tokens up to and including EOS).  Reference:
experiments/arllm/train_gsm8k_grpo.py:366-428 (TRL ``GRPOTrainer``:
num_generations groups, beta 0.04, epsilon 0.2, ``loss_type="grpo"``,
``scale_rewards="none"``, one optimisation pass per generation batch, fused
AdamW) and shared/verifier.py (the reward adapter; here any
``reward(prompt, completion, rng) -> float``).

Layout and data parallelism:

* Every trainable tensor (embedding / tied head, norms, fused QKV weight and
  bias, O, interleaved gate/up, down) is a view into one flat bf16 buffer.
  The inference runner reads the same views, so rollouts always use the
  current policy with no copy.
* The flat buffer is cut into buckets (one per decoder layer, one for the
  embedding + final norm), each padded to a multiple of ``world * 64``
  elements.  Rank r owns the r-th slice of every bucket; its fp32 master
  weights and AdamW moments are the concatenation of its slices.
* Backward writes fp32 weight gradients straight into a flat fp32 gradient
  buffer (the tcgen05 GEMM's fp32 epilogue targets the bucket view).  When the
  last gradient of a bucket is written, the bucket is reduce-scattered into
  the rank's gradient shard on a communication stream, overlapping the
  backward of earlier layers.
* The fused AdamW kernel updates the master shard (global-norm clipping with
  an all-reduced squared norm) and writes the bf16 shard, which is
  all-gathered back into the flat buffer per bucket.
"""

from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Callable

import numpy as np
import torch
import torch.nn.functional as F

from ..arllm.config import SamplingConfig
from ..arllm.types import GenerationRequest
from ..models.decoder import DecoderConfig, DecoderWeights, build_weights, random_state_dict
from ..ops import kernels as K

LAYER_FIELDS = ("in_norm", "w_qkv", "b_qkv", "q_norm", "k_norm", "w_o", "post_norm", "w_gu", "w_down")
NORM_FIELDS = ("in_norm", "post_norm", "q_norm", "k_norm", "final_norm")


@dataclass(frozen=True)
class GRPOConfig:
    group_size: int = 8
    prompts_per_rank: int = 1
    prompt_length: int = 256
    completion_length: int = 512
    learning_rate: float = 1e-6
    beta: float = 0.04
    epsilon: float = 0.2
    temperature: float = 1.0
    max_grad_norm: float = 1.0
    weight_decay: float = 0.0
    adam_betas: tuple[float, float] = (0.9, 0.999)
    adam_eps: float = 1e-8
    scale_rewards: str = "none"      # "none" | "group"
    head_chunk_rows: int = 2048
    eos_token_id: int | None = None
    seed: int = 0
    dp_collectives: str = "symmetric"   # "symmetric" (peer-memory kernels, CUDA) | "nccl"

    def __post_init__(self):
        if min(self.group_size, self.prompts_per_rank, self.prompt_length, self.completion_length,
               self.head_chunk_rows) < 1:
            raise ValueError("positive group / prompt / completion sizes required")
        if self.group_size < 2:
            raise ValueError("group-normalised advantages need at least two completions per prompt")
        if self.scale_rewards not in ("none", "group"):
            raise ValueError("scale_rewards must be none or group")
        if not (self.learning_rate > 0 and self.epsilon > 0 and self.beta >= 0 and self.max_grad_norm > 0):
            raise ValueError("positive learning rate / epsilon / clip and non-negative beta required")
        if self.dp_collectives not in ("symmetric", "nccl"):
            raise ValueError("dp_collectives must be symmetric or nccl")


def group_advantages(rewards: torch.Tensor, group: int, scale: str = "none") -> torch.Tensor:
    """r - mean(group), optionally divided by the group's standard deviation (+1e-4)."""
    r = rewards.view(-1, group).float()
    adv = r - r.mean(1, keepdim=True)
    if scale == "group":
        adv = adv / (r.std(1, keepdim=True) + 1e-4)
    return adv.reshape(-1)


class _PrecomputedGradLoss(torch.autograd.Function):
    """A scalar loss whose gradient with respect to ``logp`` was computed along with it."""

    @staticmethod
    def forward(ctx, logp, loss, grad):
        ctx.save_for_backward(grad)
        return loss.clone()

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        return grad * g, None, None


def grpo_loss(logp: torch.Tensor, old_logp: torch.Tensor, ref_logp: torch.Tensor, advantages: torch.Tensor,
              mask: torch.Tensor, *, beta: float, epsilon: float) -> tuple[torch.Tensor, dict]:
    """Clipped-ratio policy loss with a k3 KL penalty, token-mean per sequence then sequence mean.

    On the GPU one fused kernel computes the loss, its gradient and the metrics
    (``csrc/grpo.cu``); on the CPU the same expression runs in torch.  The metrics come
    back as floats: one device-to-host read of three values.
    """
    if logp.is_cuda:
        value, grad, stats = K.grpo_loss(logp, old_logp, ref_logp, advantages, mask, beta=beta, epsilon=epsilon)
        loss = _PrecomputedGradLoss.apply(logp, value, grad)
        kl, clip = stats[1:].tolist()
        return loss, {"kl": kl, "clip_fraction": clip}
    ratio = torch.exp(logp - old_logp)
    a = advantages[:, None]
    obj = torch.minimum(ratio * a, ratio.clamp(1 - epsilon, 1 + epsilon) * a)
    delta = ref_logp - logp
    kl = torch.exp(delta) - delta - 1
    m = mask.float()
    per_seq = ((obj - beta * kl) * m).sum(1) / m.sum(1).clamp(min=1)
    loss = -per_seq.mean()
    with torch.no_grad():
        clipped = ((ratio - 1).abs() > epsilon).float()
        info = {"kl": float((kl * m).sum() / m.sum()), "clip_fraction": float((clipped * m).sum() / m.sum())}
    return loss, info


# ------------------------------------------------------------ flat params --
@dataclass
class _Slot:
    offset: int
    shape: tuple[int, ...]
    bucket: int
    uses: int


class FlatParameters:
    """bf16 parameters as views of one flat buffer, bucketed and sharded over data-parallel ranks."""

    def __init__(self, named: list[tuple[str, torch.Tensor, int, int]], world: int, rank: int, device,
                 align: int = 64, allocate: Callable[[int, torch.dtype], torch.Tensor] | None = None):
        # named: (name, tensor, bucket key, uses per forward)
        self.world, self.rank = world, rank
        buckets: dict[int, list] = {}
        for name, t, b, uses in named:
            buckets.setdefault(b, []).append((name, t, uses))
        self.slots: dict[str, _Slot] = {}
        self.bucket_ranges: list[tuple[int, int]] = []
        off = 0
        quantum = world * align
        for b in sorted(buckets):
            lo = off
            for name, t, uses in buckets[b]:
                self.slots[name] = _Slot(off, tuple(t.shape), len(self.bucket_ranges), uses)
                off += -(-t.numel() // 8) * 8            # 16-byte aligned starts
            off = lo + -(-(off - lo) // quantum) * quantum
            self.bucket_ranges.append((lo, off))
        self.numel = off
        self.flat = (allocate(self.numel, torch.bfloat16) if allocate is not None
                     else torch.zeros(self.numel, dtype=torch.bfloat16, device=device))
        for name, t, _, _ in named:
            self.view(name).copy_(t)
        self.trainable = sum(t.numel() for _, t, _, _ in named)

    def view(self, name: str, buf: torch.Tensor | None = None) -> torch.Tensor:
        s = self.slots[name]
        n = math.prod(s.shape)
        return (self.flat if buf is None else buf)[s.offset:s.offset + n].view(s.shape)

    def shard_ranges(self) -> list[tuple[int, int, int]]:
        """(flat lo, flat hi, shard offset) of this rank's slice of every bucket."""
        out, pos = [], 0
        for lo, hi in self.bucket_ranges:
            n = (hi - lo) // self.world
            out.append((lo + self.rank * n, lo + (self.rank + 1) * n, pos))
            pos += n
        return out

    @property
    def shard_numel(self) -> int:
        return self.numel // self.world


class GradientSink:
    """fp32 gradient buffer whose buckets are reduce-scattered as soon as they are complete.

    ``dp`` (:mod:`online_speculation_b200.parallel.dp`) owns the gradient buffer and the
    reduce-scatter: the peer-memory kernel or NCCL; every bucket's shard is the data-parallel
    mean of the ranks' gradients.
    """

    def __init__(self, params: FlatParameters, group, device, dp=None):
        self.p = params
        self.group = group
        self.world = params.world
        self.dp = dp
        self.grad = (dp.allocate(params.numel, torch.float32) if dp is not None
                     else torch.zeros(params.numel, dtype=torch.float32, device=device))
        # one rank: the whole buffer is the shard
        self.shard = self.grad if self.world == 1 else torch.zeros(params.shard_numel, dtype=torch.float32,
                                                                   device=device)
        self.expected = [0] * len(params.bucket_ranges)
        for s in params.slots.values():
            self.expected[s.bucket] += s.uses
        self.stream = torch.cuda.Stream(device=device) if self.grad.is_cuda and self.world > 1 else None
        self._ranges = params.shard_ranges()
        self.written: set[str] = set()
        self.pending: list[int] = []
        self.launched: list[int] = []

    def begin(self) -> None:
        self.written.clear()
        self.pending = list(self.expected)
        self.launched = []

    def view(self, name: str) -> torch.Tensor:
        return self.p.view(name, self.grad)

    def write(self, name: str, fn: Callable[[torch.Tensor | None], torch.Tensor | None]) -> None:
        """``fn(out)`` computes the gradient: into ``out`` on the first use, returned (and added) after."""
        v = self.view(name)
        if name not in self.written:
            r = fn(v)
            if r is not None and r.data_ptr() != v.data_ptr():
                v.copy_(r.view_as(v))
            self.written.add(name)
        else:
            v.add_(fn(None).view_as(v))
        self._done(name)

    def add_rows(self, name: str, index: torch.Tensor, rows: torch.Tensor) -> None:
        v = self.view(name)
        if name not in self.written:
            v.zero_()
            self.written.add(name)
        v.index_add_(0, index, rows.float())
        self._done(name)

    def _done(self, name: str) -> None:
        b = self.p.slots[name].bucket
        self.pending[b] -= 1
        if self.pending[b] == 0:
            self._reduce(b)

    def _reduce(self, b: int) -> None:
        lo, hi = self.p.bucket_ranges[b]
        pos = self._ranges[b][2]
        n = (hi - lo) // self.world
        for name, s in self.p.slots.items():       # parameters without a gradient this step contribute zeros
            if s.bucket == b and name not in self.written:
                self.view(name).zero_()
                self.written.add(name)
        self.launched.append(b)
        if self.world == 1:
            return
        if self.stream is None:
            self.dp.reduce_scatter(self.grad, lo, hi, self.shard[pos:pos + n], 1.0 / self.world)
            return
        self.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.stream):
            self.dp.reduce_scatter(self.grad, lo, hi, self.shard[pos:pos + n], 1.0 / self.world)

    def finish(self) -> torch.Tensor:
        """Reduce any bucket not launched yet, wait for the reductions, return the averaged shard."""
        for b in range(len(self.pending)):
            if b not in self.launched:
                self.pending[b] = 0
                self._reduce(b)
        if self.stream is not None:
            torch.cuda.current_stream().wait_stream(self.stream)
        return self.shard


class _SinkLinear(torch.autograd.Function):
    """y = x W^T (+ b); weight / bias gradients go to the gradient sink, dX through autograd."""

    @staticmethod
    def forward(ctx, x, anchor, w, b, sink, wname, bname):
        ctx.save_for_backward(x, w)
        ctx.sink, ctx.wname, ctx.bname = sink, wname, bname
        return K.linear(x, w, bias=b)

    @staticmethod
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        gy = gy.to(torch.bfloat16).contiguous()
        gx = K.linear(gy, w.t().contiguous()) if ctx.needs_input_grad[0] else None
        gyt, xt = K.transpose_padded(gy), K.transpose_padded(x)
        ctx.sink.write(ctx.wname, lambda out: K.linear(gyt, xt, out=out, out_dtype=torch.float32))
        if ctx.bname is not None:
            ctx.sink.write(ctx.bname, lambda out: torch.sum(gy.float(), 0, out=out) if out is not None
                           else gy.float().sum(0))
        return gx, None, None, None, None, None, None


class _SinkEmbedding(torch.autograd.Function):
    """table[ids]; the row gradients are scattered into the sink."""

    @staticmethod
    def forward(ctx, anchor, table, ids, sink, name):
        ctx.save_for_backward(ids)
        ctx.sink, ctx.name = sink, name
        return table[ids]

    @staticmethod
    def backward(ctx, g):
        (ids,) = ctx.saved_tensors
        ctx.sink.add_rows(ctx.name, ids.reshape(-1), g.reshape(-1, g.shape[-1]))
        return None, None, None, None, None


def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def _rope(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = t.shape[-1] // 2
    a, b = t[..., :half].float(), t[..., half:].float()
    return torch.cat((a * cos - b * sin, b * cos + a * sin), -1).to(t.dtype)


class PolicyModel:
    """Training-time forward of the decoder over named tensors.

    With a sink, the linear layers and the embedding route their weight
    gradients into it; a dummy ``anchor`` input that requires grad keeps the
    autograd graph reaching ops whose real inputs do not.
    """

    def __init__(self, config: DecoderConfig, tensors: dict[str, torch.Tensor], inv_freq: torch.Tensor,
                 sink: GradientSink | None, chunk_rows: int):
        self.cfg = config
        self.t = tensors
        self.inv_freq = inv_freq
        self.sink = sink
        self.chunk_rows = chunk_rows
        self.anchor = torch.zeros((), device=inv_freq.device, requires_grad=True) if sink is not None else None

    def _linear(self, x, w, b=None):
        bias = None if b is None else self.t[b]
        if self.sink is None:
            return K.linear(x, self.t[w], bias=bias)
        return _SinkLinear.apply(x, self.anchor, self.t[w], bias, self.sink, w, b)

    def hidden(self, ids: torch.Tensor) -> torch.Tensor:
        c, t = self.cfg, self.t
        B, T = ids.shape
        D = c.head_dim
        qh, kvh = c.num_attention_heads, c.num_key_value_heads
        eps = c.rms_norm_eps
        if self.sink is None:
            h = t["embed"][ids]
        else:
            h = _SinkEmbedding.apply(self.anchor, t["embed"], ids, self.sink, "embed")
        ang = torch.arange(T, device=ids.device, dtype=torch.float32)[:, None] * self.inv_freq[None]
        cos, sin = ang.cos()[None, :, None], ang.sin()[None, :, None]
        for i in range(c.num_hidden_layers):
            p = f"{i}."
            x = _rms(h, t[p + "in_norm"], eps).reshape(B * T, -1)
            qkv = self._linear(x, p + "w_qkv", p + "b_qkv" if c.attention_bias else None).view(B, T, -1)
            q = qkv[..., : qh * D].view(B, T, qh, D)
            k = qkv[..., qh * D:(qh + kvh) * D].view(B, T, kvh, D)
            v = qkv[..., (qh + kvh) * D:].view(B, T, kvh, D)
            if c.qk_norm:
                q, k = _rms(q, t[p + "q_norm"], eps), _rms(k, t[p + "k_norm"], eps)
            q, k = _rope(q, cos, sin), _rope(k, cos, sin)
            att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                 is_causal=True, enable_gqa=True)
            att = att.transpose(1, 2).reshape(B * T, qh * D)
            h = h + self._linear(att, p + "w_o").view(B, T, -1)
            x = _rms(h, t[p + "post_norm"], eps).reshape(B * T, -1)
            gu = self._linear(x, p + "w_gu").view(B * T, -1, 2, 64)
            act = (F.silu(gu[:, :, 0].float()) * gu[:, :, 1].float()).to(torch.bfloat16).reshape(B * T, -1)
            h = h + self._linear(act, p + "w_down").view(B, T, -1)
        return _rms(h, t["final_norm"], eps)

    def completion_logprobs(self, ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
        """log p(ids[:, t] | ids[:, :t]) for the completion positions t >= prompt_len: [B, T - prompt_len]."""
        B, T = ids.shape
        hid = self.hidden(ids)[:, prompt_len - 1:T - 1].reshape(-1, self.cfg.hidden_size)
        tgt = ids[:, prompt_len:].reshape(-1)
        sink = None
        if self.sink is not None:
            s, name = self.sink, "embed" if self.cfg.tie_word_embeddings else "head"

            def sink(produce):
                s.write(name, produce)
        return K.head_logprob(hid, self.t["head"], tgt, chunk_rows=self.chunk_rows, sink=sink).view(B, -1)


def _named_tensors(w: DecoderWeights) -> list[tuple[str, torch.Tensor, int, int]]:
    tied = w.config.tie_word_embeddings
    out = [("embed", w.embed, 0, 2 if tied else 1), ("final_norm", w.final_norm, 0, 1)]
    if not tied:
        out.append(("head", w.head, 0, 1))
    for i, lw in enumerate(w.layers):
        for f in LAYER_FIELDS:
            t = getattr(lw, f)
            if t is not None:
                out.append((f"{i}.{f}", t, i + 1, 1))
    return out


def _tensors(w: DecoderWeights) -> dict[str, torch.Tensor]:
    out = {"embed": w.embed, "final_norm": w.final_norm, "head": w.head}
    for i, lw in enumerate(w.layers):
        for f in LAYER_FIELDS:
            t = getattr(lw, f)
            if t is not None:
                out[f"{i}.{f}"] = t
    return out


class GRPOTrainer:
    def __init__(self, model: DecoderConfig, config: GRPOConfig = GRPOConfig(), *, group=None, device=None,
                 seed: int = 0, kv_bytes: int = 8 << 30, reward_fn=None, rollouts: bool = True,
                 use_graphs: bool = True, state_dict: dict | None = None):
        self.cfg = model
        self.config = config
        self.group = group
        if group is not None:
            import torch.distributed as dist

            self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        else:
            self.world, self.rank = 1, 0
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else "cpu"
        self.device = torch.device(device)
        sd = state_dict if state_dict is not None else random_state_dict(model, seed=seed, device=self.device)
        policy = build_weights(model, sd, device=self.device)
        ref = build_weights(model, sd, device=self.device)
        del sd
        # data-parallel collectives: peer-memory kernels over symmetric buffers on GPUs, else the process group
        self.dp = None
        if self.world > 1:
            from ..parallel.dp import make_data_parallel

            kind = config.dp_collectives if self.device.type == "cuda" else "nccl"
            self.dp = make_data_parallel(group, self.device, kind)
        # flat bf16 parameters; the runner's weights become views of it
        self.params = FlatParameters(_named_tensors(policy), self.world, self.rank, self.device,
                                     allocate=None if self.dp is None else self.dp.allocate)
        self.policy_weights = self._rebind(policy)
        self.sink = GradientSink(self.params, group, self.device, dp=self.dp)
        leaves = {}
        for name in self.params.slots:
            v = self.params.view(name)
            leaves[name] = v.detach().requires_grad_(True) if name.split(".")[-1] in NORM_FIELDS else v
        leaves["head"] = leaves["embed"] if model.tie_word_embeddings else leaves["head"]
        self.leaves = leaves
        self._hook_norms()
        self.policy = PolicyModel(model, leaves, policy.inv_freq, self.sink, config.head_chunk_rows)
        self.reference = PolicyModel(model, _tensors(ref), ref.inv_freq, None, config.head_chunk_rows)
        # fp32 master shard + AdamW moments
        shard = torch.empty(self.params.shard_numel, dtype=torch.float32, device=self.device)
        for lo, hi, pos in self.params.shard_ranges():
            shard[pos:pos + hi - lo].copy_(self.params.flat[lo:hi])
        self.master = shard
        self.exp_avg = torch.zeros_like(shard)
        self.exp_avg_sq = torch.zeros_like(shard)
        self.publish = torch.empty(self.params.shard_numel, dtype=torch.bfloat16, device=self.device)
        self.sq_norm = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.nonfinite = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.backend = None
        if rollouts:
            from ..engine.backend import EngineBackend
            from ..engine.kv_cache import KVCache
            from ..engine.runner import ModelRunner

            seq_tokens = config.prompt_length + config.completion_length
            layers, kvh = model.num_hidden_layers, policy.heads.kv_slots
            cache = KVCache(layers, kvh, KVCache.pages_for_budget(kv_bytes, layers, kvh), self.device)
            batch = config.group_size * config.prompts_per_rank
            runner = ModelRunner(policy, cache, max_tokens=max(4096, seq_tokens), max_logit_rows=max(64, batch))
            self.backend = EngineBackend(runner, max_batch=batch, max_seq_tokens=seq_tokens + 64,
                                         use_graphs=use_graphs, prefix_cache_pages=0)
        self.rng = np.random.default_rng(config.seed + 1000 * self.rank)
        self.reward_fn = reward_fn or (lambda prompt, completion, rng: float(rng.random() < 0.5))
        self.step_count = 0
        self.stats: dict = {}

    # ---- parameter plumbing ----
    def _rebind(self, w: DecoderWeights) -> DecoderWeights:
        v = self.params.view
        w.embed = v("embed")
        w.final_norm = v("final_norm")
        w.head = v("embed") if self.cfg.tie_word_embeddings else v("head")
        for i, lw in enumerate(w.layers):
            for f in LAYER_FIELDS:
                if getattr(lw, f) is not None:
                    setattr(lw, f, v(f"{i}.{f}"))
        return w

    def _hook_norms(self) -> None:
        sink = self.sink

        def make(name):
            def hook(p):
                g = p.grad
                p.grad = None
                sink.write(name, lambda out: g.float())
            return hook

        for name, leaf in self.leaves.items():
            if leaf.requires_grad and name != "head":
                leaf.register_post_accumulate_grad_hook(make(name))

    def parameter(self, name: str) -> torch.Tensor:
        """Current bf16 value of a named trainable tensor (``embed``, ``final_norm``, ``3.w_qkv`` ...)."""
        return self.params.view(name)

    # ---- rollouts ----
    def rollout(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, list]:
        """Sample the group completions: (ids [B, P + C], completion mask [B, C], rewards [B], samples)."""
        if self.backend is None:
            raise RuntimeError("constructed without a rollout backend")
        c = self.config
        V = self.cfg.vocab_size
        prompts = [tuple(int(x) for x in self.rng.integers(0, V, c.prompt_length)) for _ in range(c.prompts_per_rank)]
        sampling = SamplingConfig(temperature=c.temperature, eos_token_id=c.eos_token_id)
        reqs = [GenerationRequest(p, c.completion_length, sampling, seed=int(self.rng.integers(0, 2**62)),
                                  request_id=f"grpo:{self.rank}:{self.step_count}:{i}:{g}")
                for i, p in enumerate(prompts) for g in range(c.group_size)]
        samples = self.backend.sample_batch(reqs)
        B, C = len(samples), c.completion_length
        ids = np.zeros((B, c.prompt_length + C), dtype=np.int64)
        mask = np.zeros((B, C), dtype=bool)
        for j, s in enumerate(samples):
            n = len(s.token_ids)
            ids[j, :c.prompt_length] = s.prefix
            ids[j, c.prompt_length:c.prompt_length + n] = s.token_ids
            mask[j, :n] = True
        rewards = [self.reward_fn(s.prefix, s.token_ids, self.rng) for s in samples]
        return (torch.from_numpy(ids).to(self.device), torch.from_numpy(mask).to(self.device),
                torch.tensor(rewards, dtype=torch.float32, device=self.device), samples)

    # ---- optimisation ----
    def compute_gradients(self, ids: torch.Tensor, mask: torch.Tensor, rewards: torch.Tensor
                          ) -> tuple[torch.Tensor, dict]:
        """Forward / backward of the GRPO loss; returns (this rank's averaged fp32 gradient shard, metrics)."""
        c = self.config
        adv = group_advantages(rewards, c.group_size, c.scale_rewards)
        with torch.no_grad():
            ref_lp = self.reference.completion_logprobs(ids, c.prompt_length)
        self.sink.begin()
        lp = self.policy.completion_logprobs(ids, c.prompt_length)
        loss, info = grpo_loss(lp, lp.detach(), ref_lp, adv, mask, beta=c.beta, epsilon=c.epsilon)
        loss.backward()
        g = self.sink.finish()
        return g, {"loss": float(loss.detach()), "reward_mean": float(rewards.mean()), **info}

    def train_on(self, ids: torch.Tensor, mask: torch.Tensor, rewards: torch.Tensor) -> dict:
        """One GRPO optimisation step on given rollouts (each rank passes its own)."""
        g, info = self.compute_gradients(ids, mask, rewards)
        self._optimizer_step(g)
        return info

    def _optimizer_step(self, g: torch.Tensor) -> None:
        c = self.config
        self.step_count += 1
        if g.is_cuda:
            K._ext.require().grad_sq_norm(g, self.sq_norm)
        else:
            self.sq_norm.copy_(g.square().sum().view(1))
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(self.sq_norm, group=self.group)
        if g.is_cuda:
            K._ext.require().adamw(self.master, g, self.exp_avg, self.exp_avg_sq, self.publish, self.sq_norm,
                                   float(c.max_grad_norm), float(c.learning_rate), c.adam_betas[0],
                                   c.adam_betas[1], c.adam_eps, float(c.weight_decay), self.step_count,
                                   self.nonfinite, None)
        else:
            norm = float(self.sq_norm.sqrt())
            scale = min(1.0, c.max_grad_norm / (norm + 1e-6))
            K.adamw_step(self.master, g * scale, self.exp_avg, self.exp_avg_sq, step=self.step_count,
                         lr=c.learning_rate, betas=c.adam_betas, eps=c.adam_eps, weight_decay=c.weight_decay,
                         publish=self.publish)
        if self.world > 1:
            self._gather_parameters()
        else:
            self.params.flat.copy_(self.publish)

    def _gather_parameters(self) -> None:
        """Every rank's bf16 shard into every rank's flat parameters (one collective per bucket)."""
        for (lo, hi, pos), (blo, bhi) in zip(self.params.shard_ranges(), self.params.bucket_ranges):
            self.dp.all_gather(self.params.flat, blo, bhi, self.publish[pos:pos + hi - lo])

    def step(self) -> dict:
        from ..utils.tracing import trace_range

        t0 = time.perf_counter()
        with trace_range("grpo.rollout"):
            ids, mask, rewards, _ = self.rollout()
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        t1 = time.perf_counter()
        with trace_range("grpo.train"):
            out = self.train_on(ids, mask, rewards)
        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
            from ..ops import workspace

            workspace.check_status(self.device)     # a cross-rank wait that ran out raises here
        t2 = time.perf_counter()
        out.update(tokens=int(ids.numel()), completions=int(ids.shape[0]), completion_tokens=int(mask.sum()),
                   rollout_s=t1 - t0, train_s=t2 - t1,
                   grad_norm=float(self.sq_norm.sqrt()), step=self.step_count)
        self.stats = out
        return out

    # ---- checkpointing ----
    def state_dict(self) -> dict:
        """This rank's resumable state: its fp32 master shard, AdamW moments, step and data RNG.

        The bf16 parameters are not saved: they are the all-gathered bf16 image of the
        master shards and are rebuilt on load.  The frozen reference copy is rebuilt
        from the initial weights by the caller.
        """
        return {"format": "grpo-shard-v1", "rank": self.rank, "world": self.world, "step": self.step_count,
                "shard_numel": self.params.shard_numel, "master": self.master.detach().cpu().clone(),
                "exp_avg": self.exp_avg.detach().cpu().clone(), "exp_avg_sq": self.exp_avg_sq.detach().cpu().clone(),
                "rng": self.rng.bit_generator.state}

    def load_state_dict(self, state: dict) -> None:
        """Restore :meth:`state_dict` of the same rank of a run with the same layout."""
        if state.get("format") != "grpo-shard-v1":
            raise ValueError("not a GRPO shard checkpoint")
        if (state["rank"], state["world"], state["shard_numel"]) != (self.rank, self.world, self.params.shard_numel):
            raise ValueError(f"checkpoint shard of rank {state['rank']} / {state['world']} "
                             f"({state['shard_numel']} elements) does not fit rank {self.rank} / {self.world} "
                             f"({self.params.shard_numel})")
        for name in ("master", "exp_avg", "exp_avg_sq"):
            saved = state[name]
            if saved.shape != getattr(self, name).shape or not bool(torch.isfinite(saved).all()):
                raise ValueError(f"checkpoint tensor {name} is malformed")
            getattr(self, name).copy_(saved)
        self.step_count = int(state["step"])
        self.rng.bit_generator.state = state["rng"]
        self.publish.copy_(self.master)
        if self.world > 1:
            self._gather_parameters()
        else:
            for lo, hi, pos in self.params.shard_ranges():
                self.params.flat[lo:hi].copy_(self.publish[pos:pos + hi - lo])

    def check_finite(self) -> bool:
        return int(self.nonfinite.item()) == 0

    def close(self) -> None:
        if self.backend is not None:
            self.backend.close()
