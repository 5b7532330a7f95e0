"""Python entry points of the hot ops.

Each function dispatches on the device of its inputs: CUDA tensors run the
hand-written sm_100a kernel of the compiled extension (and raise if it is
missing); CPU tensors run the plain PyTorch fp32 oracle that defines the op and
that the kernel tests compare against.  There is no other backend.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from . import _ext, workspace

PAGE_SIZE = 32
HEAD_DIM = 128


# ----------------------------------------------------------------- linear --
def linear(
    x: torch.Tensor,
    w: torch.Tensor,
    *,
    bias: torch.Tensor | None = None,
    residual: torch.Tensor | None = None,
    out: torch.Tensor | None = None,
    swiglu: bool = False,
    out_dtype: torch.dtype = torch.bfloat16,
    allow_split: bool = True,
    static_weights: bool = False,
    split_mode: int = 0,
) -> torch.Tensor:
    """``x @ w.T (+ bias) (+ residual)``; with ``swiglu`` the weight rows are
    tiles of [64 gate | 64 up] rows and the result is ``silu(gate) * up``.

    ``split_mode``: with fewer output tiles than SMs, K is split across a
    thread-block cluster reduced through distributed shared memory (0) or across
    CTAs reduced through the global fp32 workspace by the last arrival (1).

    ``residual`` may alias ``out`` (in-place residual-stream update).
    ``static_weights``: no kernel earlier in the stream writes ``w`` (inference
    weights), so the GEMM may stream weight tiles while its predecessor runs.
    """
    rows = w.shape[0] // 2 if swiglu else w.shape[0]
    if out is None:
        out = torch.empty(x.shape[0], rows, dtype=out_dtype, device=x.device)
    if x.is_cuda:
        ext = _ext.require()
        ext.gemm(
            w,
            x,
            out,
            bias,
            residual,
            1 if swiglu else 0,
            allow_split,
            workspace.gemm_workspace(x.device),
            workspace.gemm_counters(x.device),
            workspace.status(x.device),
            static_weights,
            split_mode,
        )
        return out
    out.copy_(linear_reference(x, w, bias=bias, residual=residual, swiglu=swiglu).to(out.dtype))
    return out


def linear_reference(x, w, *, bias=None, residual=None, swiglu=False):
    y = x.float() @ w.float().t()
    if bias is not None:
        y = y + bias.float()
    if swiglu:
        tiles = y.view(y.shape[0], -1, 2, 64)
        gate, up = tiles[:, :, 0, :], tiles[:, :, 1, :]
        y = (torch.nn.functional.silu(gate) * up).reshape(y.shape[0], -1)
    if residual is not None:
        y = y + residual.float()
    return y


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """Pack [F, H] gate and up weights into [2F, H] tiles of [64 gate | 64 up]."""
    features, hidden = gate.shape
    if features % 64:
        pad = 64 - features % 64
        gate = torch.cat((gate, gate.new_zeros(pad, hidden)))
        up = torch.cat((up, up.new_zeros(pad, hidden)))
    return torch.stack((gate.view(-1, 64, hidden), up.view(-1, 64, hidden)), 1).reshape(-1, hidden).contiguous()


# ---------------------------------------------------------------- rmsnorm --
def rmsnorm(x, weight, eps, *, out=None, residual=None, delta=None):
    """RMSNorm; with ``delta``: ``residual = x + delta`` (written) then norm."""
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        _ext.require().rmsnorm(x, weight, out, float(eps), residual, delta)
        return out
    src = x
    if delta is not None:
        residual.copy_((x.float() + delta.float()).to(x.dtype))
        src = residual
    work = src.float()
    normed = (work * torch.rsqrt(work.square().mean(-1, keepdim=True) + eps)).to(x.dtype)
    out.copy_(normed * weight)
    return out


# ------------------------------------------------------------------- rope --
def rope_frequencies(head_dim: int, theta: float) -> torch.Tensor:
    """Inverse frequencies, formed on the host in fp32 (as the reference does)."""
    idx = torch.arange(0, head_dim, 2, dtype=torch.float32)
    half = 1.0 / (theta ** (idx / head_dim))
    # kernel layout: element d and d + D/2 share frequency index d
    return half


def rope_cache(qkv, positions, slots, inv_freq, q_out, k_cache, v_cache, num_q, num_kv, *, q_norm=None,
               k_norm=None, eps=1e-6):
    """Split fused QKV rows, optional per-head Q/K RMSNorm, RoPE, write Q and paged K/V.

    ``k_cache``/``v_cache``: one layer, [pages, Hkv, P, D].  ``slots`` int32 [T]
    (physical slot = page * P + offset, -1 = do not store).
    """
    if qkv.is_cuda:
        _ext.require().rope_cache(qkv, positions, slots, inv_freq_full(inv_freq), q_norm, k_norm, float(eps), q_out,
                                  k_cache, v_cache, int(num_q), int(num_kv), workspace.status(qkv.device))
        return q_out
    q, k, v = rope_reference(qkv, positions, inv_freq, num_q, num_kv, q_norm=q_norm, k_norm=k_norm, eps=eps)
    q_out.copy_(q.view_as(q_out))
    page = k_cache.shape[2]
    for t in range(qkv.shape[0]):
        s = int(slots[t]) if slots is not None else -1
        if s >= 0:
            k_cache[s // page, :, s % page] = k[t]
            v_cache[s // page, :, s % page] = v[t]
    return q_out


def inv_freq_full(inv_freq: torch.Tensor) -> torch.Tensor:
    """Expand [D/2] frequencies to the [D/2] + padding layout the kernel indexes."""
    return inv_freq


def rope_reference(qkv, positions, inv_freq, num_q, num_kv, *, q_norm=None, k_norm=None, eps=1e-6):
    T = qkv.shape[0]
    D = HEAD_DIM
    q = qkv[:, : num_q * D].reshape(T, num_q, D)
    k = qkv[:, num_q * D : (num_q + num_kv) * D].reshape(T, num_kv, D)
    v = qkv[:, (num_q + num_kv) * D : (num_q + 2 * num_kv) * D].reshape(T, num_kv, D)

    def norm(x, w):
        if w is None:
            return x
        work = x.float()
        return (work * torch.rsqrt(work.square().mean(-1, keepdim=True) + eps)).to(x.dtype) * w

    q, k = norm(q, q_norm), norm(k, k_norm)
    angle = positions.float().cpu()[:, None] * inv_freq.float().cpu()[None, :]
    cos, sin = angle.cos().to(qkv.device), angle.sin().to(qkv.device)

    def rot(x):
        x = x.float()
        a, b = x[..., : D // 2], x[..., D // 2 :]
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat((a * c - b * s, b * c + a * s), -1).to(qkv.dtype)

    return rot(q), rot(k), v


# -------------------------------------------------------------- embedding --
def embed(ids, table, out=None):
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    if table.is_cuda:
        _ext.require().embed(ids, table, out, workspace.status(ids.device))
        return out
    out.copy_(table[ids.long()])
    return out


def page_copy(cache, pairs):
    """Copy (src page, dst page, tokens) triples for every layer of [L, pages, Hkv, P, D]."""
    if pairs.numel() == 0:
        return
    if cache.is_cuda:
        _ext.require().page_copy(cache, pairs)
        return
    for src, dst, count in pairs.tolist():
        cache[:, dst, :, :count] = cache[:, src, :, :count]


# -------------------------------------------------------------- attention --
@dataclass
class AttentionPlan:
    """Per-launch sequence metadata (device int32 tensors) for paged attention."""

    table: torch.Tensor
    q_start: torch.Tensor
    q_len: torch.Tensor
    kv_len: torch.Tensor
    mode: torch.Tensor
    tile_seq: torch.Tensor
    tile_row0: torch.Tensor
    tile_rows: int
    # host copies for the CPU oracle
    host: dict
    kv_splits: int = 1
    # two-pass attention over a key prefix that every sequence shares (None: one pass)
    shared: "SharedPrefix | None" = None


@dataclass
class SharedPrefix:
    """The shared-prefix pass of two-pass attention and the buffers it hands to the second pass.

    Every sequence of the batch sees the same first ``keys`` keys (the same cache pages).  The
    first pass treats the query rows of all sequences as one bidirectional block against those
    keys, so each prefix page is read once per KV head instead of once per sequence, and writes
    the normalised fp32 output and the log2-domain log-sum-exp per (token, head); the second pass
    runs each sequence over keys [keys, kv_len) and merges the first pass into its result.
    """

    plan: AttentionPlan       # one bidirectional sequence: all query tokens x the shared keys
    k_lo: torch.Tensor        # [B] int32, the first key of the per-sequence pass (= keys)
    o: torch.Tensor           # [T, Hq, D] fp32
    lse: torch.Tensor         # [T, Hq] fp32
    keys: int


def shared_prefix(table: torch.Tensor, tokens: int, keys: int, sequences: int, group: int, q_heads: int,
                  device, tile_rows: int = 32) -> SharedPrefix:
    """Plan the shared-prefix pass for ``tokens`` query tokens (row 0 of ``table`` holds the shared pages).

    ``keys`` must be a multiple of the page size; ``group`` is query heads per KV head.
    """
    if keys % PAGE_SIZE:
        raise ValueError("the shared prefix must be whole pages")
    rows = tokens * group
    tiles = -(-rows // tile_rows)
    one = lambda v: torch.tensor([v], dtype=torch.int32, device=device)
    plan = AttentionPlan(table[:1], one(0), one(tokens), one(keys), one(1),
                         torch.zeros(tiles, dtype=torch.int32, device=device),
                         torch.arange(0, tiles * tile_rows, tile_rows, dtype=torch.int32, device=device), tile_rows, {})
    return SharedPrefix(plan, torch.full((sequences,), keys, dtype=torch.int32, device=device),
                        torch.empty(tokens, q_heads, 128, dtype=torch.float32, device=device),
                        torch.empty(tokens, q_heads, dtype=torch.float32, device=device), keys)


TC_TILE_ROWS = 128          # query rows per CTA of the tcgen05 attention kernel
TC_CHUNK_KEYS = 64          # keys per pipeline chunk of that kernel
SM_COUNT = 148


def attention_kv_splits(tiles: int, max_kv: int, sms: int = SM_COUNT) -> int:
    """Key splits per tile for the tcgen05 kernel: the (tile, kv head) CTAs of one launch
    are few when sequences are few (e.g. a handful of decode rows per rank under tensor
    parallelism), so long key ranges are cut into 2, 4 or 8 pieces whose partial softmax
    states merge inside a thread-block cluster.  Every piece keeps at least two chunks."""
    splits = 1
    while splits < 8 and tiles * splits * 2 <= sms and max_kv >= 2 * splits * 2 * TC_CHUNK_KEYS:
        splits *= 2
    return splits


def attention_tile_rows(rows_per_seq: int, ctas: int, max_kv: int, sms: int = SM_COUNT) -> int:
    """Kernel choice by shape (measured on B200).  The tcgen05 kernel runs one softmax
    thread per query row of a 128-row tile, so it wins wherever tiles are full or the
    key range can be split over a cluster: prefill and diffusion (1.8-1.9x the mma.sync
    kernel), and decode / verify with few (sequence, kv head) pairs (64 x 1024 keys on
    one kv head: 17.8 vs 25.3 us; 8 x 4096: 27.5 vs 57.9 us).  Many short decode tiles
    (64 sequences x 4 kv heads x 1024 keys, 28 rows each) still run faster on the
    mma.sync kernel with TMA-fed key groups (35.8 vs 55 us), which streams four key
    groups per tile and co-schedules two tiles per SM."""
    if rows_per_seq >= 64 or attention_kv_splits(ctas, max_kv, sms) > 1:
        return TC_TILE_ROWS
    return 16 if rows_per_seq <= 16 else 32


def plan_attention(table, q_lens, kv_lens, modes, group, device, *, tile_rows=None, kv_splits=None, kv_heads=1):
    """Build the tile list of one attention launch.

    ``table``: int32 [B, max_pages] page table; ``q_lens``/``kv_lens``/``modes``:
    python lists; ``group``: query heads per kv head.  ``tile_rows`` None (default)
    chooses by shape (:func:`attention_tile_rows`): 128 is the tcgen05 kernel (128-row
    tiles, optional key splits over a cluster), 16 / 32 / 64 the mma.sync kernels.
    ``kv_heads``: KV heads of the launch (the grid's second dimension), used only to
    choose the key split.
    """
    q_start, acc = [], 0
    for n in q_lens:
        q_start.append(acc)
        acc += n
    if tile_rows is None:
        most = max(n * group for n in q_lens) if q_lens else 0
        tile_rows = attention_tile_rows(most, len(q_lens) * max(1, kv_heads), max(kv_lens) if kv_lens else 0)
    tile_seq, tile_row0 = [], []
    for b, n in enumerate(q_lens):
        rows = n * group
        for r0 in range(0, rows, tile_rows):
            tile_seq.append(b)
            tile_row0.append(r0)
    if tile_rows != TC_TILE_ROWS:
        kv_splits = 1
    elif kv_splits is None:
        kv_splits = attention_kv_splits(len(tile_seq) * max(1, kv_heads), max(kv_lens) if kv_lens else 0)

    def dev(values):
        return torch.tensor(values, dtype=torch.int32).to(device, non_blocking=True)

    host = {"q_start": q_start, "q_len": list(q_lens), "kv_len": list(kv_lens), "mode": list(modes),
            "table": table.cpu() if table.is_cuda else table}
    return AttentionPlan(table.to(device, non_blocking=True), dev(q_start), dev(list(q_lens)), dev(list(kv_lens)),
                         dev(list(modes)), dev(tile_seq), dev(tile_row0), tile_rows, host, kv_splits)


def attention(q, k_cache, v_cache, plan: AttentionPlan, *, out=None, scale=None):
    """Paged attention; ``q`` [T, Hq, D], caches [pages, Hkv, P, D] of one layer."""
    if out is None:
        out = torch.empty_like(q)
    scale = scale if scale is not None else q.shape[-1] ** -0.5
    if q.is_cuda:
        ext = _ext.require()
        st = workspace.status(q.device)
        pre = plan.shared
        if pre is None:
            ext.attention(q, k_cache, v_cache, plan.table, plan.q_start, plan.q_len, plan.kv_len, plan.mode,
                          plan.tile_seq, plan.tile_row0, plan.tile_rows, plan.kv_splits, out, float(scale), st,
                          None, None, None, None, None)
            return out
        p = pre.plan
        ext.attention(q, k_cache, v_cache, p.table, p.q_start, p.q_len, p.kv_len, p.mode, p.tile_seq, p.tile_row0,
                      p.tile_rows, 1, out, float(scale), st, None, pre.o, pre.lse, None, None)
        ext.attention(q, k_cache, v_cache, plan.table, plan.q_start, plan.q_len, plan.kv_len, plan.mode,
                      plan.tile_seq, plan.tile_row0, plan.tile_rows, plan.kv_splits, out, float(scale), st,
                      pre.k_lo, None, None, pre.o, pre.lse)
        return out
    out.copy_(attention_reference(q, k_cache, v_cache, plan.host, scale))
    return out


def gather_kv(cache, pages, length):
    """[Hkv, length, D] view of a sequence's keys or values."""
    page = cache.shape[2]
    blocks = [cache[p] for p in pages[: (length + page - 1) // page]]
    return torch.cat(blocks, 1)[:, :length]


def attention_reference(q, k_cache, v_cache, host, scale):
    out = torch.zeros(q.shape, dtype=torch.float32)
    Hq, Hkv = q.shape[1], k_cache.shape[1]
    G = Hq // Hkv
    for b, (s, n, kv, mode) in enumerate(zip(host["q_start"], host["q_len"], host["kv_len"], host["mode"])):
        pages = host["table"][b].tolist()
        k = gather_kv(k_cache.cpu(), pages, kv).float().repeat_interleave(G, 0)
        v = gather_kv(v_cache.cpu(), pages, kv).float().repeat_interleave(G, 0)
        qb = q[s : s + n].cpu().float().transpose(0, 1)  # [Hq, n, D]
        scores = (qb @ k.transpose(1, 2)) * scale
        if not mode:
            qpos = torch.arange(kv - n, kv)[:, None]
            kpos = torch.arange(kv)[None, :]
            scores = scores.masked_fill(kpos > qpos, float("-inf"))
        out[s : s + n] = (scores.softmax(-1) @ v).transpose(0, 1)
    return out.to(q.dtype).to(q.device)


# ---------------------------------------------------------------- sampling --
def sample(logits, inv_temp, uniforms, *, tokens=None, logq=None, logp=None, arith=None, next_uniforms=None,
           top_k=None, top_p=None):
    """Inverse-CDF sampling (float64 prefix sums) at per-row temperature.

    Returns (tokens int32, log q under the policy, log p at temperature one).
    With ``arith`` (int32 per row) and ``next_uniforms``, every flagged row is
    an arithmetic-coding draw: its uniform is a code point and the rescaled
    point for the next token, (u - cumulative mass before the token) / mass of
    the token, is written to ``next_uniforms``.  ``top_k`` (int32 per row, 0 =
    off) and ``top_p`` (float32 per row, 1 = off) truncate the policy
    (:func:`truncated_log_policy`); log p stays the full-support T = 1 law.
    """
    rows = logits.shape[0]
    dev = logits.device
    tokens = tokens if tokens is not None else torch.empty(rows, dtype=torch.int32, device=dev)
    logq = logq if logq is not None else torch.empty(rows, dtype=torch.float32, device=dev)
    logp = logp if logp is not None else torch.empty(rows, dtype=torch.float32, device=dev)
    if logits.is_cuda:
        _ext.require().sample(logits, inv_temp, uniforms, tokens, logq, logp, arith, next_uniforms, top_k, top_p)
        return tokens, logq, logp
    t, q, p, nxt = sample_reference(logits, inv_temp, uniforms, with_code=True, top_k=top_k, top_p=top_p)
    tokens.copy_(t)
    logq.copy_(q)
    logp.copy_(p)
    if arith is not None and next_uniforms is not None:
        flat = next_uniforms.reshape(rows, -1)[:, 0] if next_uniforms.dim() > 1 else next_uniforms
        flat.copy_(torch.where(arith.bool(), nxt, flat.double()).to(flat.dtype))
    return tokens, logq, logp


def truncated_log_policy(z, top_k=None, top_p=None):
    """log softmax of tempered logits ``z`` [rows, V] under per-row top-k / top-p truncation (fp32 oracle).

    top-k keeps every column at least as large as the k-th largest; top-p then sorts
    the kept columns in descending order and keeps each one whose preceding mass
    (renormalised over the kept set) is at most top_p, the rule of
    src/inference_scaling/arllm/backends/transformers_backend.py:323-348.
    ``top_k`` / ``top_p`` are per-row tensors (0 / 1 disable a row's filter) or None.
    """
    z = z.float().clone()
    rows, V = z.shape
    if top_k is not None:
        k = top_k.to(torch.long).cpu().tolist()
        for r in range(rows):
            if 0 < k[r] < V:
                kth = torch.topk(z[r], k[r]).values[-1]
                z[r] = z[r].masked_fill(z[r] < kth, float("-inf"))
    if top_p is not None:
        p = top_p.float().cpu().tolist()
        for r in range(rows):
            if p[r] < 1.0:
                ordered, order = torch.sort(z[r], descending=True)
                mass = torch.softmax(ordered, -1)
                drop = mass.cumsum(-1) > p[r]
                drop = torch.cat((drop.new_zeros(1), drop[:-1]))
                z[r] = z[r].masked_fill(torch.zeros_like(drop).scatter(0, order, drop), float("-inf"))
    return z.log_softmax(-1)


def sample_reference(logits, inv_temp, uniforms, *, with_code=False, top_k=None, top_p=None):
    x = logits.float()
    it = inv_temp.float()[:, None] if inv_temp is not None else torch.ones(x.shape[0], 1, device=x.device)
    log_q = truncated_log_policy(x * it, top_k, top_p)
    log_p = x.log_softmax(-1)
    mass = log_q.exp().double()
    cumulative = mass.cumsum(-1)
    cumulative[:, -1] = 1.0
    u = uniforms.reshape(x.shape[0], -1)[:, 0].double()
    tok = (cumulative < u[:, None]).sum(-1).clamp_max(x.shape[1] - 1)
    out = (tok.int(), log_q.gather(-1, tok[:, None]).squeeze(-1), log_p.gather(-1, tok[:, None]).squeeze(-1))
    if not with_code:
        return out
    m = mass.gather(-1, tok[:, None]).squeeze(-1)
    lo = cumulative.gather(-1, tok[:, None]).squeeze(-1) - m
    nxt = ((u - lo) / m.clamp_min(1e-300)).clamp(0.0, 0.99999999999999989)
    return out + (nxt,)


def row_stats(logits, inv_temp=None, targets=None, *, top_k=None, top_p=None):
    """Per-row lse at T=1 and at T, plus log p / log q of ``targets`` (scoring).

    With ``top_k`` / ``top_p`` (per-row tensors) lse at T and log q are those of
    the truncated policy; a target outside the kept columns gets log q = -inf.
    """
    rows, dev = logits.shape[0], logits.device
    lse1 = torch.empty(rows, dtype=torch.float32, device=dev)
    lseT = torch.empty(rows, dtype=torch.float32, device=dev)
    logp = torch.empty(rows, dtype=torch.float32, device=dev) if targets is not None else None
    logq = torch.empty(rows, dtype=torch.float32, device=dev) if targets is not None else None
    if logits.is_cuda:
        _ext.require().row_stats(logits, inv_temp, targets, lse1, lseT, logp, logq,
                                 *workspace.row_stats_split(dev), top_k, top_p)
        return lse1, lseT, logp, logq
    x = logits.float()
    it = inv_temp.float()[:, None] if inv_temp is not None else torch.ones(rows, 1)
    z = x * it
    lse1.copy_(torch.logsumexp(x, -1))
    if top_k is None and top_p is None:
        lseT.copy_(torch.logsumexp(z, -1))
        log_q = z - lseT[:, None]
    else:
        log_q = truncated_log_policy(z, top_k, top_p)
        kept = torch.isfinite(log_q)
        lseT.copy_(torch.where(kept, z - log_q, torch.full_like(z, float("-inf"))).amax(-1))
    if targets is not None:
        idx = targets.long()[:, None]
        logp.copy_(x.gather(-1, idx).squeeze(-1) - lse1)
        logq.copy_(log_q.gather(-1, idx).squeeze(-1))
    return lse1, lseT, logp, logq


HEAD_STATS_ROWS = 8192   # rows per head-statistics launch (bounds the partial buffer)


def head_stats(x, weight, inv_temp=None, targets=None):
    """Row statistics of ``x @ weight.T`` without storing the logits (vocabulary-head scoring).

    ``x`` [R, H] bf16 (already normalised), ``weight`` [V, H] bf16.  Returns fp32
    (lse at T = 1, lse at T, log p of ``targets`` at T = 1, log q at T); the last
    two are None without targets.  On the GPU the tcgen05 GEMM reduces every
    128-row vocabulary tile to (max, sum exp, sum exp at 1/T) in its epilogue and
    one warp per row folds the tiles; rows go in chunks of ``HEAD_STATS_ROWS``.
    """
    R, V = x.shape[0], weight.shape[0]
    dev = x.device
    lse1 = torch.empty(R, dtype=torch.float32, device=dev)
    lseT = torch.empty(R, dtype=torch.float32, device=dev)
    logp = torch.empty(R, dtype=torch.float32, device=dev) if targets is not None else None
    logq = torch.empty(R, dtype=torch.float32, device=dev) if targets is not None else None
    if not x.is_cuda:
        logits = x.float() @ weight.float().t()
        a, b, c, d = row_stats(logits, inv_temp, targets)
        lse1.copy_(a)
        lseT.copy_(b)
        if targets is not None:
            logp.copy_(c)
            logq.copy_(d)
        return lse1, lseT, logp, logq
    ext = _ext.require()
    tiles = -(-V // 128)
    chunk = min(R, HEAD_STATS_ROWS)
    part = workspace.scratch(dev, "head_stats_part", chunk * tiles * 4, torch.float32)
    tlogit = workspace.scratch(dev, "head_stats_target", chunk, torch.float32)
    status = workspace.status(dev)
    it = inv_temp.float().contiguous() if inv_temp is not None else None
    tg = targets.to(torch.int32).contiguous() if targets is not None else None
    for s in range(0, R, chunk):
        e = min(R, s + chunk)
        ext.head_stats(weight, x[s:e], None if it is None else it[s:e], None if tg is None else tg[s:e], part,
                       tlogit, lse1[s:e], lseT[s:e], None if logp is None else logp[s:e],
                       None if logq is None else logq[s:e], status)
    return lse1, lseT, logp, logq


def remask_select(tokens, a0, bl, mask_id, drawn, tc, *, prio=None, logq=None, subset=False, traj=None,
                  pos_offset=0):
    """One block-diffusion remasking step, in place on ``tokens`` [B, S] (int64).

    Among the masked positions of block [a0, a0 + bl) every row commits the ``tc``
    with the highest ``prio`` [B * bl] (ties: lower position; None: earliest first)
    to its ``drawn`` [B * bl] token.  Returns (chosen positions + ``pos_offset`` in
    increasing order [B, tc], chosen tokens [B, tc], the step's log density [B] in
    float64 or None without ``logq``); ``traj`` [B] float64 accumulates the density,
    plus log 1 / C(masked, tc) with ``subset``.
    """
    B = tokens.shape[0]
    dev = tokens.device
    out_pos = torch.empty(B, tc, dtype=torch.int64, device=dev)
    out_tok = torch.empty(B, tc, dtype=torch.int64, device=dev)
    step_lp = torch.empty(B, dtype=torch.float64, device=dev) if logq is not None else None
    if tokens.is_cuda:
        _ext.require().remask_select(tokens, int(a0), int(bl), int(mask_id), drawn.to(torch.int32).contiguous(),
                                     None if prio is None else prio.float().contiguous(),
                                     None if logq is None else logq.float().contiguous(), int(tc), bool(subset),
                                     traj, step_lp, out_pos, out_tok, int(pos_offset))
        return out_pos, out_tok, step_lp
    masked = tokens[:, a0:a0 + bl] == mask_id
    positions = torch.arange(bl, device=dev)
    p = (-positions.float()).expand(B, bl) if prio is None else prio.view(B, bl).float()
    p = p.masked_fill(~masked, float("-inf"))
    # rank by (priority descending, position ascending)
    order = torch.argsort(-p, dim=1, stable=True)
    sel = order[:, :tc].sort(dim=1).values
    chosen = drawn.view(B, bl).long().gather(1, sel)
    tokens[:, a0:a0 + bl].scatter_(1, sel, chosen)
    out_pos.copy_(sel + pos_offset)
    out_tok.copy_(chosen)
    if logq is not None:
        lp = logq.view(B, bl).double().gather(1, sel).sum(1)
        if subset:
            n = masked.sum(1).double()
            lp = lp - (torch.lgamma(n + 1) - math.lgamma(tc + 1) - torch.lgamma(n - tc + 1))
        step_lp.copy_(lp)
        if traj is not None:
            traj += lp
    return out_pos, out_tok, step_lp


@dataclass
class VocabShard:
    """This rank's slice [v_lo, v_lo + width) of a vocabulary of v_total columns (tensor parallel).

    Samplers given a shard scan only the local logits and exchange per-row
    scalars (packed argmax keys, log-normalisers, candidate logits) through
    small collectives instead of gathering full logits rows.
    """

    v_lo: int
    width: int
    v_total: int
    group: object
    world: int

    def __post_init__(self):
        self._bufs: dict = {}

    def buf(self, name, shape, dtype, device):
        key = (name, tuple(shape), dtype)
        t = self._bufs.get(key)
        if t is None:
            t = self._bufs[key] = torch.zeros(shape, dtype=dtype, device=device)
        return t

    def all_reduce(self, t, op="sum"):
        import torch.distributed as dist

        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM, group=self.group)
        return t

    def logsumexp(self, local: torch.Tensor) -> torch.Tensor:
        """Global log-normalisers from per-rank ones ([..] -> [..])."""
        import torch.distributed as dist

        flat = local.reshape(-1)
        gathered = self.buf("lse_gather", (self.world, flat.numel()), flat.dtype, flat.device)
        dist.all_gather_into_tensor(gathered, flat.contiguous(), group=self.group)
        return torch.logsumexp(gathered, 0).view_as(local)


_ORD_NEG_INF = 0x007FFFFF   # monotone bit pattern of -inf in the packed argmax keys


def unpack_argmax_keys(keys: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Packed (score, column) keys -> (column int64, found bool)."""
    k = keys ^ torch.iinfo(torch.int64).min
    col = 0xFFFFFFFF - (k & 0xFFFFFFFF)
    found = ((k >> 32) & 0xFFFFFFFF) != _ORD_NEG_INF
    return col, found


def gumbel_sample(logits, inv_temp, seeds, *, seed_index=None, streams=None, row_in_seq=None, salt=0, tokens=None,
                  shard: VocabShard | None = None):
    """Gumbel-max (exponential race) sampling with counter-based randomness.

    With ``shard``, ``logits`` holds this rank's vocabulary columns; every rank
    returns the same global token (noise is keyed by the global column)."""
    rows = logits.shape[0]
    tokens = tokens if tokens is not None else torch.empty(rows, dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        best, count = workspace.sampler_split(logits.device)
    if logits.is_cuda and shard is not None:
        keys = shard.buf("gumbel_keys", (rows,), torch.int64, logits.device)
        _ext.require().gumbel_sample(logits, inv_temp, seeds, seed_index, streams, row_in_seq, int(salt), tokens,
                                     shard.v_lo, keys, best, count)
        shard.all_reduce(keys, "max")
        tokens.copy_(unpack_argmax_keys(keys)[0])
        return tokens
    if logits.is_cuda:
        _ext.require().gumbel_sample(logits, inv_temp, seeds, seed_index, streams, row_in_seq, int(salt), tokens,
                                     0, None, best, count)
        return tokens
    x = logits.float() * (inv_temp.float()[:, None] if inv_temp is not None else 1.0)
    if seed_index is None and streams is None and row_in_seq is None:
        gen = torch.Generator().manual_seed(int(seeds.flatten()[0]) ^ int(salt))
        e = torch.empty_like(x).exponential_(generator=gen)
    else:
        # per-row streams keyed like the device kernel's counters (row-independent draws)
        e = torch.empty_like(x)
        flat = seeds.flatten().tolist()
        for r in range(rows):
            sd = flat[int(seed_index[r])] if seed_index is not None else flat[0]
            key = (int(sd) * 1000003 + (int(streams[r]) if streams is not None else 0)) * 1000003
            key = (key + (int(row_in_seq[r]) if row_in_seq is not None else r)) ^ int(salt)
            gen = torch.Generator().manual_seed(key % (2**63))
            e[r].exponential_(generator=gen)
    tokens.copy_((x.softmax(-1) / e).argmax(-1))
    return tokens


def spec_verify(target, draft, candidates, inv_temp, seeds, *, streams=None, salt=0, out=None, stats=None,
                shard: VocabShard | None = None):
    """Exact p/q correction of a batch of draft blocks.

    ``target`` [B*(n+1), V] logits, ``draft`` [B*n, V] logits, ``candidates`` [B, n].
    Returns dict of count, tail, valid, emitted [B, n+1], logq, logp [B, n+1].
    On CUDA the row log-normalisers are first computed by the row-parallel
    statistics kernel (one CTA per row); ``stats`` may hold preallocated
    buffers (``inv_target`` [B*(n+1)], ``inv_draft`` [B*n], ``lse1_t``,
    ``lseT_t``, ``lse1_d``, ``lseT_d``) for graph capture.
    """
    B, n = candidates.shape
    dev = target.device
    res = out or {
        "count": torch.empty(B, dtype=torch.int32, device=dev),
        "tail": torch.empty(B, dtype=torch.int32, device=dev),
        "valid": torch.empty(B, dtype=torch.int32, device=dev),
        "emitted": torch.empty(B, n + 1, dtype=torch.int32, device=dev),
        "logq": torch.empty(B, n + 1, dtype=torch.float32, device=dev),
        "logp": torch.empty(B, n + 1, dtype=torch.float32, device=dev),
    }
    if target.is_cuda:
        ext = _ext.require()
        if stats is None:
            it = inv_temp if inv_temp is not None else torch.ones(B, dtype=torch.float32, device=dev)
            stats = {"inv_target": it.repeat_interleave(n + 1), "inv_draft": it.repeat_interleave(n),
                     "lse1_t": torch.empty(B * (n + 1), dtype=torch.float32, device=dev),
                     "lseT_t": torch.empty(B * (n + 1), dtype=torch.float32, device=dev),
                     "lse1_d": torch.empty(B * n, dtype=torch.float32, device=dev),
                     "lseT_d": torch.empty(B * n, dtype=torch.float32, device=dev)}
        split = workspace.row_stats_split(target.device)
        ext.row_stats(target, stats["inv_target"], None, stats["lse1_t"], stats["lseT_t"], None, None, *split, None,
                      None)
        ext.row_stats(draft, stats["inv_draft"], None, stats["lse1_d"], stats["lseT_d"], None, None, *split, None,
                      None)
        if shard is not None:
            return _spec_verify_shard(target, draft, candidates, inv_temp, seeds, streams, salt, res, stats, shard)
        ext.spec_verify(target, draft, candidates, n, inv_temp, seeds, streams, int(salt), res["count"],
                        res["tail"], res["valid"], res["emitted"], res["logq"], res["logp"], stats["lseT_t"],
                        stats["lse1_t"], stats["lseT_d"], 0, 0, None, None)
        return res
    gen = torch.Generator().manual_seed(int(seeds.flatten()[0]) ^ int(salt))
    for b in range(B):
        it = float(inv_temp[b]) if inv_temp is not None else 1.0
        p = (target[b * (n + 1) : (b + 1) * (n + 1)].float() * it).softmax(-1)
        q = (draft[b * n : (b + 1) * n].float() * it).softmax(-1)
        count = n
        for i in range(n):
            x = int(candidates[b, i])
            if not float(torch.rand((), generator=gen)) < min(1.0, float(p[i, x] / q[i, x])):
                count = i
                break
        if count < n:
            resid = (p[count] - q[count]).clamp_min(0)
            tail = int(torch.multinomial(resid / resid.sum(), 1, generator=gen))
        else:
            tail = int(torch.multinomial(p[n], 1, generator=gen))
        emitted = candidates[b, :count].tolist() + [tail]
        res["count"][b], res["tail"][b], res["valid"][b] = count, tail, 1
        lt = target[b * (n + 1) : (b + 1) * (n + 1)].float()
        for i, x in enumerate(emitted):
            res["emitted"][b, i] = x
            res["logq"][b, i] = (lt[i] * it).log_softmax(-1)[x]
            res["logp"][b, i] = lt[i].log_softmax(-1)[x]
    return res


def _spec_verify_shard(target, draft, candidates, inv_temp, seeds, streams, salt, res, stats, shard: VocabShard):
    """Vocabulary-parallel p/q correction: the same draws as the unsharded kernel.

    Exchanges per rank: one all-gather of the row log-normalisers, one sum of
    the candidates' logits (each owned by one rank), one max of the packed tail
    keys and one sum of the tail token's logit.
    """
    B, n = candidates.shape
    dev = target.device
    lse = torch.cat((stats["lse1_t"], stats["lseT_t"], stats["lseT_d"]))
    g = shard.logsumexp(lse)
    R = B * (n + 1)
    lse1_t, lseT_t, lseT_d = g[:R], g[R:2 * R], g[2 * R:]
    cand = candidates.long()
    local = cand - shard.v_lo
    own = (local >= 0) & (local < shard.width)
    lc = local.clamp(0, shard.width - 1)
    t_rows = (torch.arange(B, device=dev)[:, None] * (n + 1) + torch.arange(n, device=dev)[None, :])
    d_rows = (torch.arange(B, device=dev)[:, None] * n + torch.arange(n, device=dev)[None, :])
    cl = shard.buf("spec_cand", (B, n, 2), torch.float32, dev)
    cl[..., 0] = torch.where(own, target[t_rows, lc], 0.0)
    cl[..., 1] = torch.where(own, draft[d_rows, lc], 0.0)
    shard.all_reduce(cl)
    keys = shard.buf("spec_keys", (B,), torch.int64, dev)
    _ext.require().spec_verify(target, draft, candidates, n, inv_temp, seeds, streams, int(salt), res["count"],
                               res["tail"], res["valid"], res["emitted"], res["logq"], res["logp"], lseT_t, lse1_t,
                               lseT_d, shard.v_lo, shard.v_total, cl, keys)
    shard.all_reduce(keys, "max")
    tail, found = unpack_argmax_keys(keys)
    count = res["count"].long()
    row = torch.arange(B, device=dev) * (n + 1) + count
    tl_local = tail - shard.v_lo
    t_own = (tl_local >= 0) & (tl_local < shard.width)
    tv = shard.buf("spec_tail", (B,), torch.float32, dev)
    tv.copy_(torch.where(t_own, target[row, tl_local.clamp(0, shard.width - 1)], 0.0))
    shard.all_reduce(tv)
    valid = (res["valid"] != 0) & found
    tail = torch.where(valid, tail, 0)
    res["valid"].copy_(valid.int())
    res["tail"].copy_(tail.int())
    i = torch.arange(n + 1, device=dev)[None, :]
    is_tail = i == count[:, None]
    cand_pad = torch.cat((cand, torch.zeros(B, 1, dtype=torch.long, device=dev)), 1)
    logit_pad = torch.cat((cl[..., 0], torch.zeros(B, 1, device=dev)), 1)
    emitted = torch.where(is_tail, tail[:, None], cand_pad)
    logit = torch.where(is_tail, tv[:, None], logit_pad)
    it = inv_temp[:, None] if inv_temp is not None else 1.0
    keep = i <= count[:, None]
    res["emitted"].copy_(torch.where(keep, emitted, 0).int())
    res["logq"].copy_(torch.where(keep, logit * it - lseT_t.view(B, n + 1), 0.0))
    res["logp"].copy_(torch.where(keep, logit - lse1_t.view(B, n + 1), 0.0))
    return res


# ------------------------------------------------------------------- grpo --
def grpo_loss_reference(logp, old_logp, ref_logp, advantages, mask, *, beta, epsilon):
    """fp32 oracle of the GRPO loss: (loss, per-token dLoss/dlogp, [loss, token-mean KL, clip fraction]).

    Per token min(r A, clip(r, 1 - eps, 1 + eps) A) - beta (exp(ref - lp) - (ref - lp) - 1) with
    r = exp(lp - old), token mean per sequence, mean over sequences, negated; the gradient
    comes from autograd of exactly that expression.
    """
    lp = logp.detach().float().clone().requires_grad_(True)
    ratio = torch.exp(lp - old_logp.float())
    a = advantages.float()[:, None]
    obj = torch.minimum(ratio * a, ratio.clamp(1 - epsilon, 1 + epsilon) * a)
    delta = ref_logp.float() - lp
    kl = torch.exp(delta) - delta - 1
    m = mask.float()
    per_seq = ((obj - beta * kl) * m).sum(1) / m.sum(1).clamp(min=1)
    loss = -per_seq.mean()
    (grad,) = torch.autograd.grad(loss, lp)
    with torch.no_grad():
        tokens = m.sum().clamp(min=1)
        clipped = ((ratio - 1).abs() > epsilon).float()
        stats = torch.stack((loss.detach(), (kl * m).sum() / tokens, (clipped * m).sum() / tokens))
    return loss.detach(), grad, stats


def grpo_loss(logp, old_logp, ref_logp, advantages, mask, *, beta, epsilon):
    """Fused GRPO loss on the GPU (one launch): returns (loss [], dLoss/dlogp [B, C], stats [3]).

    ``stats`` = (loss, token-mean KL, clipped-token fraction), left on the device.  CPU
    tensors take :func:`grpo_loss_reference`.
    """
    if not logp.is_cuda:
        return grpo_loss_reference(logp, old_logp, ref_logp, advantages, mask, beta=beta, epsilon=epsilon)
    B, C = logp.shape
    dev = logp.device
    lp, old, ref = (t.detach().float().contiguous() for t in (logp, old_logp, ref_logp))
    grad = torch.empty_like(lp)
    rows = torch.empty(B, 4, dtype=torch.float32, device=dev)
    out = torch.empty(3, dtype=torch.float32, device=dev)
    # zero when created; the kernel's last block resets it after every launch
    counter = workspace.zeros(dev, "grpo_counter", 1, torch.int32)
    _ext.require().grpo_loss(lp, old, ref, advantages.detach().float().contiguous(), mask.contiguous(),
                             float(beta), float(epsilon), grad, rows, out, counter)
    return out[0], grad, out


# ------------------------------------------------------------------ adamw --
def adamw_step(params, grads, exp_avg, exp_avg_sq, *, step, lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0,
               clip=None, publish=None, norm_out=None, nonfinite=None, step_tensor=None):
    """Fused AdamW on flat fp32 buffers with global-norm clipping; optional bf16 publish.

    ``step_tensor`` (int32 [1] on the device) supplies the step for the bias
    corrections instead of ``step``, so the update can be replayed from a graph.
    """
    if params.is_cuda:
        ext = _ext.require()
        sq = None
        if clip is not None:
            sq = norm_out if norm_out is not None else torch.empty(1, dtype=torch.float32, device=params.device)
            ext.grad_sq_norm(grads, sq)
        ext.adamw(params, grads, exp_avg, exp_avg_sq, publish, sq, float(clip or 0.0), float(lr), float(betas[0]),
                  float(betas[1]), float(eps), float(weight_decay), int(step), nonfinite, step_tensor)
        return sq
    scale = 1.0
    sq = grads.float().square().sum()
    if clip is not None:
        norm = float(sq.sqrt())
        if not math.isfinite(norm):
            if nonfinite is not None:
                nonfinite.fill_(1)
            return sq
        scale = min(1.0, clip / (norm + 1e-6))
    g = grads * scale
    params.mul_(1 - lr * weight_decay)
    exp_avg.mul_(betas[0]).add_(g, alpha=1 - betas[0])
    exp_avg_sq.mul_(betas[1]).addcmul_(g, g, value=1 - betas[1])
    if step_tensor is not None:
        step = int(step_tensor.flatten()[0])
    bc1, bc2 = 1 - betas[0] ** step, 1 - betas[1] ** step
    params.addcdiv_(exp_avg / bc1, (exp_avg_sq / bc2).sqrt().add_(eps), value=-lr)
    if publish is not None:
        publish.copy_(params)
    return sq


# ------------------------------------------------- head + distillation loss --
class _HeadDivergence(torch.autograd.Function):
    """Per-row TV / forward-KL between softmax(y @ W^T) and softmax(teacher).

    Forward: tcgen05 GEMM to fp32 logits, then the fused statistics and loss
    kernels (two passes over the logits).  Backward: one kernel writes
    d loss / d logits in bf16, then d y = d logits @ W.  Under a
    vocabulary-sharded head the row statistics and loss pieces are all-reduced
    across ranks between the phases.
    """

    @staticmethod
    def forward(ctx, y, weight, teacher, kind, comm):
        ext = _ext.require()
        R = y.shape[0]
        logits = linear(y.to(torch.bfloat16).contiguous(), weight, out_dtype=torch.float32)
        stats = torch.empty(R, 4, dtype=torch.float32, device=y.device)
        ext.divergence_stats(logits, teacher, stats)
        world = 1 if comm is None else comm.world
        if world > 1:
            import torch.distributed as dist

            m = stats[:, 0::2].contiguous()
            dist.all_reduce(m, op=dist.ReduceOp.MAX, group=comm.group)
            sums = stats[:, 1::2] * torch.exp(stats[:, 0::2] - m)
            dist.all_reduce(sums, group=comm.group)
            lse = (m + sums.log()).contiguous()
        else:
            lse = (stats[:, 0::2] + stats[:, 1::2].log()).contiguous()
        pieces = torch.empty(R, 2, dtype=torch.float32, device=y.device)
        ext.divergence_loss(logits, teacher, lse, int(kind), pieces)
        if world > 1:
            import torch.distributed as dist

            dist.all_reduce(pieces, group=comm.group)
        ctx.save_for_backward(logits, teacher, lse, pieces, weight)
        ctx.kind = int(kind)
        return pieces[:, 0].clone()

    @staticmethod
    def backward(ctx, g):
        logits, teacher, lse, pieces, weight = ctx.saved_tensors
        grad = torch.empty(logits.shape, dtype=torch.bfloat16, device=logits.device)
        _ext.require().divergence_grad(logits, teacher, lse, pieces, g.float().contiguous(), ctx.kind, grad)
        dy = (grad @ weight).float()
        return dy, None, None, None, None


def head_divergence(y: torch.Tensor, weight: torch.Tensor, teacher: torch.Tensor, kind: str = "tv", comm=None):
    """Per-row divergence of the head logits of ``y`` [R, H] from ``teacher`` [R, V_local] logits."""
    k = 0 if kind == "tv" else 1
    if y.is_cuda:
        return _HeadDivergence.apply(y, weight, teacher, k, comm)
    log_q = (y.float() @ weight.float().t()).log_softmax(-1)
    log_p = teacher.float().log_softmax(-1)
    if k == 0:
        return 0.5 * (log_q.exp() - log_p.exp()).abs().sum(-1)
    return (log_p.exp() * (log_p - log_q)).sum(-1)


# ------------------------------------------------ training-time autograd ops --
def transpose_padded(a: torch.Tensor, multiple: int = 8) -> torch.Tensor:
    """``a.t()`` as a contiguous tensor whose row length is zero-padded to ``multiple`` elements.

    The tcgen05 GEMM reads K-major operands through TMA, whose row stride must
    be a multiple of 16 bytes; weight gradients reduce over the token
    dimension, which becomes the row length after the transpose.
    """
    rows, cols = a.shape
    padded = -(-rows // multiple) * multiple
    if padded == rows:
        return a.t().contiguous()
    out = torch.zeros(cols, padded, dtype=a.dtype, device=a.device)
    out[:, :rows].copy_(a.t())
    return out


class _KernelLinear(torch.autograd.Function):
    """y = x @ w^T (+ b) on the tcgen05 GEMM, with a tcgen05 backward.

    dX = dY @ W runs as dY @ (W^T)^T with a transposed copy of W (cached per
    weight version); dW = dY^T @ X runs as (dY^T) @ (X^T)^T with transposed
    activations.  Both are ordinary K-major problems for the same kernel.
    """

    @staticmethod
    def forward(ctx, x, w, b, w_t, need_wgrad):
        ctx.save_for_backward(x, w, w_t)
        ctx.has_bias = b is not None
        ctx.need_wgrad = need_wgrad
        return linear(x, w, bias=b)

    @staticmethod
    def backward(ctx, gy):
        x, w, w_t = ctx.saved_tensors
        gy = gy.to(torch.bfloat16).contiguous()
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            wt = w_t if w_t is not None else w.t().contiguous()
            gx = linear(gy, wt)
        if ctx.need_wgrad:
            gw = linear(transpose_padded(gy), transpose_padded(x), out_dtype=torch.float32)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gb = gy.float().sum(0)
        return gx, gw, gb, None, None


def kernel_linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None, *, w_t: torch.Tensor | None = None,
                  weight_grad: bool = True) -> torch.Tensor:
    """Autograd linear on the sm_100a GEMM (CUDA) or PyTorch (CPU).

    ``weight_grad=True`` returns an fp32 gradient for ``w`` (for fp32 masters)."""
    shape = x.shape
    x2 = x.reshape(-1, shape[-1]).to(torch.bfloat16).contiguous()
    if x.is_cuda:
        y = _KernelLinear.apply(x2, w, b, w_t, weight_grad and w.requires_grad)
    else:
        y = torch.nn.functional.linear(x2.float(), w.float(), None if b is None else b.float()).to(torch.bfloat16)
    return y.reshape(*shape[:-1], w.shape[0])


class _TargetLogprob(torch.autograd.Function):
    """log softmax(logits)[target] per row with the fused statistics / gradient kernels."""

    @staticmethod
    def forward(ctx, logits, targets):
        ext = _ext.require()
        R = logits.shape[0]
        lse1 = torch.empty(R, dtype=torch.float32, device=logits.device)
        lseT = torch.empty_like(lse1)
        logp = torch.empty_like(lse1)
        logq = torch.empty_like(lse1)
        ext.row_stats(logits, None, targets, lse1, lseT, logp, logq, *workspace.row_stats_split(logits.device),
                      None, None)
        ctx.save_for_backward(logits, lse1, targets)
        return logp

    @staticmethod
    def backward(ctx, g):
        logits, lse, targets = ctx.saved_tensors
        grad = torch.empty_like(logits)
        _ext.require().logprob_grad(logits, lse, targets, g.float().contiguous(), grad)
        return grad, None


def target_logprob(logits: torch.Tensor, targets: torch.Tensor) -> torch.Tensor:
    """Differentiable per-row log-probability of ``targets`` under softmax(logits) (fp32 rows)."""
    if logits.is_cuda:
        return _TargetLogprob.apply(logits.float().contiguous(), targets.to(torch.int32).contiguous())
    return logits.float().log_softmax(-1).gather(-1, targets.long()[:, None]).squeeze(-1)


class _HeadLogprob(torch.autograd.Function):
    """Per-row log softmax(h @ W^T)[target] over row chunks, without keeping [rows x V] logits.

    Forward: per chunk, fp32 logits from the tcgen05 GEMM and the fused row
    statistics (logsumexp, target log-probability).  Backward: per chunk the
    logits are recomputed, one kernel writes ``g (onehot - softmax)`` in bf16
    into a [rows x V] buffer, and d h = d logits @ W; finally one GEMM forms
    d W = d logits^T @ h.  With ``sink`` the weight gradient is not returned
    through autograd: ``sink(produce)`` is called with a function that
    writes d W into a given fp32 [V, H] tensor (or allocates one for None).
    """

    @staticmethod
    def forward(ctx, h, weight, targets, chunk, sink):
        R, V = h.shape[0], weight.shape[0]
        logp = torch.empty(R, dtype=torch.float32, device=h.device)
        lse = torch.empty_like(logp)
        buf = torch.empty(min(chunk, R) * V, dtype=torch.float32, device=h.device)
        for s in range(0, R, chunk):
            e = min(R, s + chunk)
            logits = linear(h[s:e], weight, out=buf[: (e - s) * V].view(e - s, V), out_dtype=torch.float32)
            if h.is_cuda:
                _ext.require().row_stats(logits, None, targets[s:e], lse[s:e], None, logp[s:e], None,
                                         *workspace.row_stats_split(logits.device), None, None)
            else:
                lse[s:e] = logits.logsumexp(-1)
                logp[s:e] = logits.gather(-1, targets[s:e].long()[:, None]).squeeze(-1) - lse[s:e]
        ctx.save_for_backward(h, weight, targets, lse)
        ctx.chunk, ctx.sink = chunk, sink
        return logp

    @staticmethod
    def backward(ctx, g):
        h, weight, targets, lse = ctx.saved_tensors
        R, V = h.shape[0], weight.shape[0]
        g = g.float().contiguous()
        glogits = torch.empty(R, V, dtype=torch.bfloat16, device=h.device)
        buf = torch.empty(min(ctx.chunk, R) * V, dtype=torch.float32, device=h.device)
        w_t = weight.t().contiguous()
        gh = torch.empty_like(h)
        for s in range(0, R, ctx.chunk):
            e = min(R, s + ctx.chunk)
            logits = linear(h[s:e], weight, out=buf[: (e - s) * V].view(e - s, V), out_dtype=torch.float32)
            if h.is_cuda:
                _ext.require().logprob_grad(logits, lse[s:e], targets[s:e], g[s:e], glogits[s:e])
            else:
                p = torch.exp(logits - lse[s:e, None])
                onehot = torch.zeros_like(p).scatter_(1, targets[s:e].long()[:, None], 1.0)
                glogits[s:e] = (g[s:e, None] * (onehot - p)).to(torch.bfloat16)
            linear(glogits[s:e], w_t, out=gh[s:e])
        del buf, w_t
        gt, ht = transpose_padded(glogits), transpose_padded(h)
        del glogits

        def produce(out):
            return linear(gt, ht, out=out, out_dtype=torch.float32)

        if ctx.sink is not None:
            ctx.sink(produce)
            return gh, None, None, None, None
        return gh, produce(None), None, None, None


def head_logprob(h: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor, *, chunk_rows: int = 2048,
                 sink=None) -> torch.Tensor:
    """log softmax(h @ weight^T)[targets] per row (fp32), differentiable in ``h`` and ``weight``."""
    return _HeadLogprob.apply(h.to(torch.bfloat16).contiguous(), weight, targets.to(torch.int32).contiguous(),
                              int(chunk_rows), sink)


# --------------------------------------------------------------------- MoE --
class MoEBuffers:
    """Static device buffers of one MoE layer invocation (reused across layers and steps)."""

    def __init__(self, max_tokens: int, experts: int, top_k: int, hidden: int, ffn: int, device):
        self.T, self.E, self.k, self.H, self.F = max_tokens, experts, top_k, hidden, ffn
        rows = max_tokens * top_k
        i32 = dict(dtype=torch.int32, device=device)
        self.logits = torch.empty(max_tokens, experts, dtype=torch.float32, device=device)
        self.idx = torch.empty(rows, **i32)
        self.w = torch.empty(rows, dtype=torch.float32, device=device)
        self.counts = torch.zeros(experts, **i32)
        self.offsets = torch.zeros(experts + 1, **i32)
        self.cursor = torch.zeros(experts, **i32)
        self.slot_of = torch.empty(rows, **i32)
        self.xp = torch.empty(rows, hidden, dtype=torch.bfloat16, device=device)
        self.act = torch.empty(rows, ffn, dtype=torch.bfloat16, device=device)
        self.y = torch.empty(rows, hidden, dtype=torch.bfloat16, device=device)
        self.total = torch.zeros(2, **i32)
        self.bn = 256
        tiles_m = max(2 * ffn, hidden) // 128
        cap = tiles_m * (-(-rows // 32) + experts)
        self.tiles = torch.zeros(2, cap * 4, **i32)


def moe_pick_bn(rows: int, experts: int) -> int:
    """Token tile of the grouped expert GEMMs from the mean rows per expert."""
    mean = rows / max(1, experts)
    return 32 if mean <= 32 else 64 if mean <= 64 else 128 if mean <= 160 else 256


def moe_ffn(x: torch.Tensor, h: torch.Tensor, router: torch.Tensor, w_gu: torch.Tensor, w_down: torch.Tensor, *,
            top_k: int, renorm: bool = False, buffers: MoEBuffers | None = None) -> torch.Tensor:
    """h += sum_j w_j * expert_{e_j}(x) for the top-k experts of every row of x (in place).

    ``router`` [E, H]; ``w_gu`` [E * 2F, H] with each expert's gate/up rows
    interleaved in 64-row tiles; ``w_down`` [E * H, F].  Routing, dispatch,
    the per-expert tile list and the combine run on the device: no host
    synchronisation between the router and the expert GEMMs.
    """
    T, H = x.shape
    E = router.shape[0]
    F = w_down.shape[1]
    if T == 0:
        return h
    if not x.is_cuda:
        return _moe_ffn_reference(x, h, router, w_gu, w_down, top_k, renorm)
    b = buffers
    if b is None or b.T < T or b.E != E or b.k != top_k or b.H != H or b.F != F:
        b = MoEBuffers(T, E, top_k, H, F, x.device)
    ext = _ext.require()
    rows = T * top_k
    logits = linear(x, router, out=b.logits[:T], out_dtype=torch.float32)
    ext.moe_route(logits, top_k, renorm, b.idx[:rows], b.w[:rows], b.counts)
    ext.moe_offsets(b.counts, b.offsets, b.cursor)
    ext.moe_dispatch(x, b.idx[:rows], b.cursor, b.xp, b.slot_of[:rows])
    bn = moe_pick_bn(rows, E)
    ws, ctr, st = workspace.gemm_workspace(x.device), workspace.gemm_counters(x.device), workspace.status(x.device)
    tm_gu, tm_dn = 2 * F // 128, H // 128
    ext.grouped_tiles(b.offsets, E, tm_gu, bn, b.tiles[0], b.total[0:1])
    ext.grouped_gemm(w_gu, b.xp[:rows], b.act[:rows], 1, b.tiles[0], b.total[0:1], E, bn, ws, ctr, st)
    if tm_dn != tm_gu:
        ext.grouped_tiles(b.offsets, E, tm_dn, bn, b.tiles[1], b.total[1:2])
        tiles, total = b.tiles[1], b.total[1:2]
    else:
        tiles, total = b.tiles[0], b.total[0:1]
    ext.grouped_gemm(w_down, b.act[:rows], b.y[:rows], 0, tiles, total, E, bn, ws, ctr, st)
    ext.moe_combine(b.y[:rows], b.slot_of[:rows], b.w[:rows], h, True)
    return h


def moe_route_reference(x: torch.Tensor, router: torch.Tensor, top_k: int, renorm: bool):
    probs = (x.float() @ router.float().t()).softmax(-1)
    # stable top-k: larger probability first, ties to the lower expert id
    order = torch.sort(-probs, dim=-1, stable=True).indices[:, :top_k]
    w = probs.gather(-1, order)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return order, w


def _moe_ffn_reference(x, h, router, w_gu, w_down, top_k, renorm):
    E = router.shape[0]
    F = w_down.shape[1]
    H = x.shape[1]
    idx, w = moe_route_reference(x, router, top_k, renorm)
    xf = x.float()
    out = torch.zeros(x.shape[0], H, dtype=torch.float32, device=x.device)
    for e in range(E):
        rows, slot = (idx == e).nonzero(as_tuple=True)
        if rows.numel() == 0:
            continue
        gu = linear_reference(x[rows], w_gu[e * 2 * F:(e + 1) * 2 * F], swiglu=True).to(torch.bfloat16)
        y = (gu.float() @ w_down[e * H:(e + 1) * H].float().t()).to(torch.bfloat16).float()
        out.index_add_(0, rows, y * w[rows, slot][:, None])
    h.copy_((h.float() + out).to(h.dtype))
    return h


def score_stats(logits: torch.Tensor, inv_temp: torch.Tensor | None, targets: torch.Tensor | None,
                topk: int = 0) -> torch.Tensor:
    """[rows, 4]: target log p at T, sum p log p, mean log p over the vocabulary, -(mean top-K log p)."""
    rows, V = logits.shape
    out = torch.empty(rows, 4, dtype=torch.float32, device=logits.device)
    if logits.is_cuda:
        _ext.require().score_stats(logits, inv_temp, None if targets is None else targets.to(torch.int32).contiguous(),
                                   int(topk), out)
        return out
    x = logits.float() * (inv_temp.float()[:, None] if inv_temp is not None else 1.0)
    lp = x.log_softmax(-1)
    out[:, 0] = lp.gather(-1, targets.long()[:, None]).squeeze(-1) if targets is not None else 0.0
    out[:, 1] = (lp.exp() * lp).sum(-1)
    out[:, 2] = lp.mean(-1)
    out[:, 3] = -lp.topk(topk, -1).values.mean(-1) if topk > 0 else 0.0
    return out
