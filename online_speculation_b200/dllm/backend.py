"""Block-wise masked-diffusion backend on the sm_100a engine (the LLaDA backend's counterpart).

Behaviour of src/inference_scaling/dllm/backends/llada.py:505-721:
for every block of ``block_length`` positions and every step of its transfer
schedule the model predicts all positions bidirectionally; a token is drawn
per masked position (argmax at T = 0, else an exponential race at temperature
T); ``transfer_count`` still-masked positions of the current block are
committed, chosen by confidence (``low_confidence``: log-probability at T = 1
of the drawn token), uniformly at random (``random``) or left to right
(``sequential``).  The mask token is excluded from the policy, top-k / top-p
filters apply before sampling, CFG combines conditional and prompt-masked
logits as u + (s + 1)(c - u).  With random / sequential remasking at T > 0
the trace carries exact step log-probabilities, including log 1/C(n, k) for
the random subset, and ``score_trajectories`` re-scores a trace under another
policy (temperature) by replaying it.

B200 design:
* the model returns logits only for the current block's rows (``rows``),
  not for every position of the sequence;
* all rows of a request group are batched; drawing, confidences, position
  selection and commits are device tensor ops (Philox-keyed Gumbel noise per
  request / step / position, so a request's draw does not depend on its batch
  neighbours); the trace is copied to the host once per group;
* ``model`` is anything with ``logits(tokens [B, L], rows [B, R]) -> fp32
  [B, R, V]``: the MoE engine (``models.moe.MoEDiffusionModel``) or, on CPU,
  a PyTorch module wrapped by :class:`ModuleLogits`.
"""

from __future__ import annotations

import threading
import time
from collections import defaultdict
from dataclasses import dataclass
from math import lgamma
from typing import Any, Sequence

import numpy as np
import torch

from ..ops import kernels as K
from .config import DiffusionSamplingConfig
from .types import (DiffusionGenerationRequest, DiffusionSample, DiffusionTraceStep,
                    DiffusionTrajectoryScoreRequest)

_GUMBEL_SALT = 0x5EED_D1FF


@dataclass(frozen=True, slots=True)
class DiffusionBackendSnapshot:
    sample_requests: int
    score_requests: int
    forward_calls: int
    model_sequences: int
    model_token_slots: int
    generated_tokens: int
    elapsed_seconds: float
    total_parameters: int
    active_parameters: int
    resident_parameters: int
    sample_forward_calls: int
    score_forward_calls: int
    sample_model_token_slots: int
    score_model_token_slots: int

    @property
    def estimated_active_flops(self) -> float:
        return 2.0 * self.active_parameters * self.model_token_slots

    @property
    def estimated_total_parameter_flops(self) -> float:
        return 2.0 * self.total_parameters * self.model_token_slots


class ModuleLogits:
    """Adapter: a PyTorch module returning full-sequence logits -> the ``logits(tokens, rows)`` contract."""

    def __init__(self, module, *, mask_token_id: int | None = None):
        self.module = module
        self.mask_token_id = mask_token_id if mask_token_id is not None else getattr(
            getattr(module, "config", None), "mask_token_id", None)

    def logits(self, tokens: torch.Tensor, rows: torch.Tensor | None = None, layer_limit: int | None = None):
        out = self.module(tokens)
        full = getattr(out, "logits", out).float()
        if rows is None:
            return full
        return full.gather(1, rows[..., None].expand(-1, -1, full.shape[-1]).to(full.device))


def subset_logprob(available: int, selected: int) -> float:
    """log 1 / C(available, selected)."""
    if not 0 <= selected <= available:
        raise ValueError("invalid subset size")
    return -(lgamma(available + 1) - lgamma(selected + 1) - lgamma(available - selected + 1))


def filter_logits(logits: torch.Tensor, sampling: DiffusionSamplingConfig) -> torch.Tensor:
    """Top-k then top-p (nucleus) filtering in place semantics of the reference policy."""
    if sampling.top_k > 0:
        kept = min(sampling.top_k, logits.shape[-1])
        thr = torch.topk(logits, kept, dim=-1).values[..., -1:]
        logits = logits.masked_fill(logits < thr, float("-inf"))
    if sampling.top_p < 1:
        sl, si = torch.sort(logits, descending=True, dim=-1)
        cum = torch.cumsum(torch.softmax(sl.float(), -1), -1)
        drop = cum > sampling.top_p
        drop[..., 1:] = drop[..., :-1].clone()
        drop[..., 0] = False
        logits = logits.masked_fill(torch.zeros_like(drop).scatter(-1, si, drop), float("-inf"))
    return logits


class DiffusionEngineBackend:
    """``DiffusionBackend`` over a bidirectional logits provider."""

    def __init__(self, model: Any, *, model_id: str | None = None, mask_token_id: int | None = None,
                 max_batch_size: int | None = None, layer_limit: int | None = None,
                 parameter_counts: tuple[int, int] | None = None, device=None):
        if max_batch_size is not None and max_batch_size <= 0:
            raise ValueError("max_batch_size must be positive when provided")
        self.model = model
        self._model_id = model_id or getattr(model, "name", None) or type(model).__name__
        mask = mask_token_id if mask_token_id is not None else getattr(model, "mask_token_id", None)
        if mask is None:
            raise ValueError("mask_token_id is absent from the model; provide it explicitly")
        self._mask = int(mask)
        self.max_batch_size = max_batch_size
        self.layer_limit = layer_limit
        self.device = torch.device(device) if device is not None else getattr(model, "device", torch.device("cpu"))
        counts = parameter_counts
        if counts is None and hasattr(model, "cfg") and hasattr(model.cfg, "parameter_counts"):
            counts = model.cfg.parameter_counts()
        self._total, self._active = counts if counts is not None else (0, 0)
        self._lock = threading.Lock()
        self._stats = defaultdict(float)

    @property
    def model_id(self) -> str:
        return self._model_id

    @property
    def mask_token_id(self) -> int:
        return self._mask

    def with_prefix_layers(self, layer_count: int) -> "DiffusionEngineBackend":
        """Early-exit proposal backend running the first ``layer_count`` layers on the same resident weights."""
        n = getattr(getattr(self.model, "cfg", None), "num_hidden_layers", None)
        if n is not None and not 0 < layer_count <= n:
            raise ValueError("layer_limit must lie within the decoder layer count")
        return DiffusionEngineBackend(self.model, model_id=f"{self.model_id}#prefix-layers={layer_count}",
                                      mask_token_id=self._mask, max_batch_size=self.max_batch_size,
                                      layer_limit=layer_count, device=self.device)

    def snapshot(self) -> DiffusionBackendSnapshot:
        s = self._stats
        return DiffusionBackendSnapshot(
            int(s["sample_requests"]), int(s["score_requests"]), int(s["forward_calls"]), int(s["model_sequences"]),
            int(s["token_slots"]), int(s["generated_tokens"]), float(s["elapsed"]), int(self._total),
            int(self._active), int(self._total), int(s["sample_forward_calls"]), int(s["score_forward_calls"]),
            int(s["sample_token_slots"]), int(s["score_token_slots"]))

    # ------------------------------------------------------------- logits --
    def _logits(self, tokens: torch.Tensor, rows: torch.Tensor, prompt_len: int, sampling: DiffusionSamplingConfig,
                phase: str) -> torch.Tensor:
        """Policy logits [B, R, V] (fp32): CFG combine, mask token excluded, top-k / top-p applied."""
        mask = self._mask
        kw = {} if self.layer_limit is None else {"layer_limit": self.layer_limit}
        if sampling.cfg_scale > 0:
            uncond = tokens.clone()
            uncond[:, :prompt_len] = mask
            if getattr(self.model, "hidden_guidance", False):
                # guidance combined on the normalised hidden rows: one vocabulary GEMM
                logits = self.model.logits(torch.cat((tokens, uncond)), torch.cat((rows, rows)),
                                           guidance=float(sampling.cfg_scale), **kw)
            else:
                both = self.model.logits(torch.cat((tokens, uncond)), torch.cat((rows, rows)), **kw)
                c, u = both.chunk(2)
                logits = u + (sampling.cfg_scale + 1.0) * (c - u)
            seqs = 2 * tokens.shape[0]
        else:
            logits = self.model.logits(tokens, rows, **kw)
            seqs = tokens.shape[0]
        logits = logits.float()
        logits[..., mask] = float("-inf")
        with self._lock:
            st = self._stats
            st["forward_calls"] += 1
            st["model_sequences"] += seqs
            st["token_slots"] += seqs * tokens.shape[1]
            st[f"{phase}_forward_calls"] += 1
            st[f"{phase}_token_slots"] += seqs * tokens.shape[1]
        return filter_logits(logits, sampling)

    # ------------------------------------------------------------- sample --
    def sample_batch(self, requests: Sequence[DiffusionGenerationRequest]) -> list[DiffusionSample]:
        if not requests:
            return []
        t0 = time.perf_counter()
        groups = defaultdict(list)
        for i, r in enumerate(requests):
            groups[(len(r.prefix), r.generation_length, r.sampling)].append((i, r))
        out: list[DiffusionSample | None] = [None] * len(requests)
        with torch.inference_mode():
            for group in groups.values():
                n = self.max_batch_size or len(group)
                for s in range(0, len(group), n):
                    chunk = group[s:s + n]
                    for (i, _), smp in zip(chunk, self._sample_group([r for _, r in chunk])):
                        out[i] = smp
        with self._lock:
            self._stats["sample_requests"] += len(requests)
            self._stats["generated_tokens"] += sum(r.generation_length for r in requests)
            self._stats["elapsed"] += time.perf_counter() - t0
        return out  # type: ignore[return-value]

    def _sample_group(self, reqs: list[DiffusionGenerationRequest]) -> list[DiffusionSample]:
        sp = reqs[0].sampling
        if sp.remasking == "low_confidence_dynamic":
            raise ValueError("dynamic-threshold remasking is not implemented by this backend")
        dev = self.device
        B, P, G = len(reqs), len(reqs[0].prefix), reqs[0].generation_length
        bl, mask = sp.block_length, self._mask
        tokens = torch.full((B, P + G), mask, dtype=torch.long, device=dev)
        if P:
            tokens[:, :P] = torch.tensor([r.prefix for r in reqs], dtype=torch.long, device=dev)
        exact = sp.has_exact_trajectory_density
        schedule = sp.transfer_schedule()
        seeds = torch.tensor([r.seed for r in reqs], dtype=torch.int64, device=dev)
        seed_index = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(bl)
        row_in = torch.arange(bl, dtype=torch.int32, device=dev).repeat(B)
        hosts = [np.random.default_rng([r.seed, 0x52414E44]) for r in reqs]   # subset priorities
        inv_t = None if sp.temperature == 0 else torch.full((B * bl,), 1.0 / sp.temperature, device=dev)
        arange_bl = torch.arange(bl, device=dev)
        rec_pos, rec_tok, rec_lp = [], [], []
        step_global = 0
        traj = torch.zeros(B, dtype=torch.float64, device=dev)
        for blk in range(G // bl):
            a0 = P + blk * bl
            rows = (a0 + arange_bl).expand(B, bl)
            for tc in schedule:
                logits = self._logits(tokens, rows, P, sp, "sample").reshape(B * bl, -1)
                if sp.temperature == 0:
                    drawn = logits.argmax(-1).to(torch.int32)
                else:
                    streams = torch.full((B * bl,), step_global, dtype=torch.int32, device=dev)
                    drawn = K.gumbel_sample(logits, inv_t, seeds, seed_index=seed_index, streams=streams,
                                            row_in_seq=row_in, salt=_GUMBEL_SALT)
                _, _, logp1, logq = K.row_stats(logits, inv_t, drawn)
                if sp.remasking in ("low_confidence", "low_confidence_static"):
                    prio = logp1                                             # most confident first
                elif sp.remasking == "random":
                    prio = torch.from_numpy(np.stack([h.random(bl) for h in hosts])).to(dev, torch.float32)
                else:
                    prio = None                                              # earliest position first
                # one fused step: choose, commit, compact and score the transferred positions
                pos, chosen, lp = K.remask_select(tokens, a0, bl, mask, drawn, tc, prio=prio,
                                                  logq=logq if exact else None, subset=sp.remasking == "random",
                                                  traj=traj if exact else None, pos_offset=blk * bl)
                if exact:
                    rec_lp.append(lp)
                rec_pos.append(pos)
                rec_tok.append(chosen)
                step_global += 1
        # one device -> host copy of the whole trace
        pos_h = torch.cat(rec_pos, 1).cpu().numpy()
        tok_h = torch.cat(rec_tok, 1).cpu().numpy()
        lp_h = torch.stack(rec_lp, 1).cpu().numpy() if exact else None
        cont = tokens[:, P:].cpu().numpy()
        samples = []
        for b, r in enumerate(reqs):
            trace, off = [], 0
            for k in range(step_global):
                tc = schedule[k % len(schedule)]
                trace.append(DiffusionTraceStep(k // len(schedule), k % len(schedule),
                                                tuple(int(v) for v in pos_h[b, off:off + tc]),
                                                tuple(int(v) for v in tok_h[b, off:off + tc]),
                                                float(lp_h[b, k]) if exact else None))
                off += tc
            samples.append(DiffusionSample(tuple(r.prefix), tuple(int(v) for v in cont[b]), tuple(trace),
                                           float(sum(s.logprob for s in trace)) if exact else None, sp.policy_id,
                                           self.model_id, r.request_id))
        return samples

    # -------------------------------------------------------------- score --
    def score_trajectories(self, requests: Sequence[DiffusionTrajectoryScoreRequest]) -> list[float]:
        if not requests:
            return []
        t0 = time.perf_counter()
        groups = defaultdict(list)
        for i, r in enumerate(requests):
            groups[(len(r.sample.prefix), len(r.sample.token_ids), r.sampling)].append((i, r))
        out: list[float | None] = [None] * len(requests)
        with torch.inference_mode():
            for group in groups.values():
                n = self.max_batch_size or len(group)
                for s in range(0, len(group), n):
                    chunk = group[s:s + n]
                    for (i, _), v in zip(chunk, self._score_group([r for _, r in chunk])):
                        out[i] = v
        with self._lock:
            self._stats["score_requests"] += len(requests)
            self._stats["elapsed"] += time.perf_counter() - t0
        return [float(v) for v in out]  # type: ignore[arg-type]

    def _score_group(self, reqs: list[DiffusionTrajectoryScoreRequest]) -> list[float]:
        sp = reqs[0].sampling
        if not sp.has_exact_trajectory_density:
            raise ValueError("trajectory scoring requires random or sequential remasking and positive temperature")
        P, G = len(reqs[0].sample.prefix), len(reqs[0].sample.token_ids)
        sp.validate_generation_length(G, prefix_length=P)
        steps = sp.total_steps(G)
        schedule = sp.transfer_schedule()
        for r in reqs:
            if len(r.sample.trace) != steps:
                raise ValueError("sample trace does not match the target transition schedule")
        dev, mask, B = self.device, self._mask, len(reqs)
        tokens = torch.full((B, P + G), mask, dtype=torch.long, device=dev)
        if P:
            tokens[:, :P] = torch.tensor([r.sample.prefix for r in reqs], dtype=torch.long, device=dev)
        totals = torch.zeros(B, dtype=torch.float64, device=dev)
        inv_t = None
        for k in range(steps):
            blk, st = divmod(k, sp.steps_per_block)
            lo, hi = blk * sp.block_length, (blk + 1) * sp.block_length
            tc = schedule[st]
            pos, tok = [], []
            for r in reqs:
                step = r.sample.trace[k]
                if step.block_index != blk or step.step_index != st:
                    raise ValueError("sample trace steps are out of schedule order")
                if len(step.positions) != tc:
                    raise ValueError("sample trace committed the wrong number of positions")
                if any(not lo <= p < hi for p in step.positions):
                    raise ValueError("sample trace committed a position outside its block")
                pos.append(step.positions)
                tok.append(step.token_ids)
            rel = torch.tensor(pos, dtype=torch.long, device=dev)
            absolute = rel + P
            if not bool((tokens.gather(1, absolute) == mask).all()):
                raise ValueError("sample trace commits an already visible position")
            avail = (tokens[:, P + lo:P + hi] == mask).sum(1)
            chosen = torch.tensor(tok, dtype=torch.long, device=dev)
            logits = self._logits(tokens, absolute, P, sp, "score").reshape(B * tc, -1)
            if inv_t is None or inv_t.numel() != B * tc:
                inv_t = torch.full((B * tc,), 1.0 / sp.temperature, device=dev)
            _, _, _, logq = K.row_stats(logits, inv_t, chosen.reshape(-1).to(torch.int32))
            lp = logq.view(B, tc).double().sum(1)
            if sp.remasking == "random":
                lp = lp + _subset_tensor(avail, tc)
            totals += lp
            tokens.scatter_(1, absolute, chosen)
        final = tokens[:, P:].cpu().numpy()
        for b, r in enumerate(reqs):
            if tuple(int(v) for v in final[b]) != tuple(r.sample.token_ids):
                raise ValueError("sample trace does not reconstruct its final continuation")
        return totals.cpu().tolist()


def _subset_tensor(available: torch.Tensor, selected: int) -> torch.Tensor:
    n = available.double()
    k = float(selected)
    return -(torch.lgamma(n + 1) - lgamma(k + 1) - torch.lgamma(n - k + 1))


__all__ = ["DiffusionBackendSnapshot", "DiffusionEngineBackend", "ModuleLogits", "filter_logits", "subset_logprob"]
