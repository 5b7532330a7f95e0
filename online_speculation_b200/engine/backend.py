"""``AutoregressiveBackend`` on the sm_100a engine: paged KV, prefix cache, graphed decode.

The B200-native counterpart of the reference's ``TransformersBackend``
(src/inference_scaling/arllm/backends/transformers_backend.py:84-1609) with
the same contract (:mod:`online_speculation_b200.arllm.types`):

* ``sample_batch`` returns, per request, the sampled tokens, their
  log-probabilities under the request's policy (temperature T) and under the
  reference policy (temperature 1, full support) from the same logits.  Token
  uniforms come from ``np.random.default_rng(seed).random(max_new_tokens)``
  (or the request's explicit ``uniforms``) and tokens are drawn by inverse CDF
  over a float64 prefix sum, exactly as the reference draws them, so a
  request's tokens do not depend on what it is batched with.  A request with
  an ``arithmetic_uniform`` is decoded by arithmetic coding: the sampler
  rescales the code point on the device after every token (cumulative mass in
  vocabulary order), so the whole sequence is a deterministic function of one
  uniform.
* ``score_batch`` packs many continuations into shared prefill forwards and
  scores their rows with the head GEMM's row-statistics epilogue (log-sum-exp at
  T = 1 and at the requested temperature plus the target logit), so no logits
  row is stored.  Top-k / top-p policies are sampled and scored with the
  truncated-policy path of the sampler kernels (radix-selected per-row
  threshold), as in the reference's policy log-softmax.

Prefix reuse: full 32-token pages are keyed by a chained hash of their tokens
and kept (reference-counted) in a prefix cache, so requests that share a
prompt -- and suffix-MH proposals that regenerate after a cut -- reuse the KV of
every cached full page instead of recomputing it.  Only the uncached remainder
is prefilled, in one packed batch.

Rollout-reuse speculation (``speculation=ActiveBatchSpeculationConfig``): a
:class:`~online_speculation_b200.arllm.acceleration.RolloutTokenTree` observes every
finished sample; when the call's batch is small enough for its tier, each request
gets a draft continuation from the tree, and all drafts of the call are verified in
ONE packed forward (last prompt token + draft, logits of every draft row) followed by
one sampler launch over those rows.  A deterministic draft token is kept only when it
equals the token the request's own uniform draws at that position, so the output law
is the target policy's; a stochastic draft is accepted with min(1, p / q) and a
rejection is redrawn from the normalised residual (p - q)+.  The KV of rejected draft
positions is truncated and decoding continues from the first unverified position
(reference: transformers_backend.py:468-642 and :1091-1224).
"""

from __future__ import annotations

import hashlib
import math
import threading
from collections import OrderedDict
from collections.abc import Sequence
from dataclasses import dataclass

import numpy as np
import torch

from ..arllm.acceleration import ActiveBatchSpeculationConfig, DraftProposal, RolloutTokenTree
from ..arllm.config import SamplingConfig
from ..arllm.types import GenerationRequest, ScoreRequest, SequenceSample
from ..ops import kernels as K
from ..shared.rng import SeedStream
from ..utils.tracing import trace_range
from .kv_cache import PAGE, KVCache
from .runner import ModelRunner, StepMeta, build_meta

BASE_POLICY = SamplingConfig().policy_id


@dataclass(frozen=True, slots=True)
class SequenceScoreStatistics:
    """Statistics of one scored continuation under a full-support policy."""

    token_logprobs: tuple[float, ...]
    mean_logprob: float
    mean_negative_entropy: float
    mean_self_certainty: float
    token_topk_confidences: tuple[float, ...] = ()
    confidence_top_k: int | None = None
BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 192, 256)


def draft_acceptance(draft: Sequence[int], sampled: Sequence[int], room: int, eos: int | None
                     ) -> tuple[int, int, bool]:
    """(tokens kept, draft tokens accepted, ended by EOS) of one verified draft.

    ``sampled[j]`` is the target's draw at draft position j (one entry more than
    ``draft``: the position after the whole draft).  Draws are kept while they equal
    the draft; the first differing draw is kept as well, and when the whole draft
    matches, the draw after it follows.  EOS and the request's remaining budget
    ``room`` end the run early.
    """
    limit = min(len(draft), room)
    accepted = 0
    for j in range(limit):
        tok = int(sampled[j])
        match = tok == int(draft[j])
        accepted += match
        if eos is not None and tok == eos:
            return j + 1, accepted, True
        if not match:
            return j + 1, accepted, False
    if limit < room:
        return limit + 1, accepted, eos is not None and int(sampled[limit]) == eos
    return limit, accepted, False


class PrefixCache:
    """Full KV pages keyed by chained token hashes, with LRU eviction.

    The cache owns one reference on every cached page; evicting drops it.
    """

    def __init__(self, cache: KVCache, max_pages: int):
        self.cache = cache
        self.max_pages = max_pages
        self._pages: OrderedDict[bytes, int] = OrderedDict()
        self.hits = 0
        self.lookups = 0

    @staticmethod
    def keys(tokens: Sequence[int], n_pages: int) -> list[bytes]:
        out, h = [], b""
        arr = np.asarray(tokens, dtype=np.int64)
        for j in range(n_pages):
            h = hashlib.blake2b(h + arr[j * PAGE:(j + 1) * PAGE].tobytes(), digest_size=16).digest()
            out.append(h)
        return out

    def lookup(self, tokens: Sequence[int], limit: int) -> tuple[list[int], list[bytes]]:
        """Cached leading full pages of ``tokens`` (at most ``limit`` tokens worth)."""
        n = min(len(tokens), limit) // PAGE
        keys = self.keys(tokens, n)
        pages = []
        for k in keys:
            p = self._pages.get(k)
            if p is None:
                break
            self._pages.move_to_end(k)
            pages.append(p)
        self.lookups += 1
        self.hits += len(pages)
        return pages, keys

    def insert(self, keys: list[bytes], pages: list[int]) -> None:
        mgr = self.cache.manager
        for k, p in zip(keys, pages):
            if k in self._pages:
                self._pages.move_to_end(k)
                continue
            mgr.retain(p)
            self._pages[k] = p
        self.evict(0)

    def evict(self, need_free: int) -> None:
        mgr = self.cache.manager
        while self._pages and (len(self._pages) > self.max_pages or mgr.free_pages < need_free):
            _, p = self._pages.popitem(last=False)
            mgr.drop(p)

    def clear(self) -> None:
        self.evict(1 << 62)


@dataclass
class _Active:
    index: int
    request: GenerationRequest
    seq: int
    last: int                 # token to feed next (its KV is not written yet)
    pos: int                  # its position
    uniforms: np.ndarray
    tokens: list
    logq: list
    logp: list
    finish: str = "length"
    carry: float | None = None     # arithmetic-coding code point for the next token


class _DecodeGraph:
    """Static buffers (+ captured graph) of S chained decode steps for B rows.

    Step s reads its input ids from row s of ``ids`` and the sampler writes the
    drawn token into row s + 1, so one replay decodes S tokens per row with a
    single host round trip.  Positions, KV slots, KV lengths and the sampling
    uniforms of all S steps are uploaded before the replay.
    """

    def __init__(self, backend: "EngineBackend", B: int, S: int, use_graph: bool):
        r = backend.runner
        dev = r.device
        self.B, self.S = B, S
        self.mp = backend.max_pages
        sizes = (B, S * B, S * B, S * B, B * self.mp)   # ids0, pos, slots, kv, table
        self.host = torch.zeros(sum(sizes), dtype=torch.int32).pin_memory()
        self.dev = torch.zeros_like(self.host, device=dev)
        hn, d = self.host.numpy(), self.dev
        o = np.cumsum((0,) + sizes)
        self.h_ids = hn[o[0]:o[1]]
        self.h_pos, self.h_slots, self.h_kv = (hn[o[k]:o[k + 1]].reshape(S, B) for k in (1, 2, 3))
        self.h_table = hn[o[4]:o[5]].reshape(B, self.mp)
        self.ids = torch.zeros(S + 1, B, dtype=torch.int32, device=dev)
        self.ids0 = d[o[0]:o[1]]
        self.pos, self.slots, self.kv = (d[o[k]:o[k + 1]].view(S, B) for k in (1, 2, 3))
        self.table = d[o[4]:o[5]].view(B, self.mp)
        self.uni_host = torch.zeros(S, B, dtype=torch.float64).pin_memory()
        # row S receives the code point after the last step of arithmetic-coding rows
        self.uni = torch.zeros(S + 1, B, dtype=torch.float64, device=dev)
        self.arith_host = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.arith = torch.zeros(B, dtype=torch.int32, device=dev)
        self.carry_host = torch.zeros(B, dtype=torch.float64).pin_memory()
        self.it_host = torch.ones(B, dtype=torch.float32).pin_memory()
        self.inv_temp = torch.ones(B, dtype=torch.float32, device=dev)
        # truncated policies per row (0 / 1 = off); the sampler reads them every step
        self.topk_host = torch.zeros(B, dtype=torch.int32).pin_memory()
        self.topp_host = torch.ones(B, dtype=torch.float32).pin_memory()
        self.top_k = torch.zeros(B, dtype=torch.int32, device=dev)
        self.top_p = torch.ones(B, dtype=torch.float32, device=dev)
        G = r.q_slots // r.kv_slots
        tr = K.attention_tile_rows(G, B * r.kv_slots, self.mp * K.PAGE_SIZE)
        tiles = -(-G // tr)
        q_start = torch.arange(B, dtype=torch.int32, device=dev)
        q_len = torch.ones(B, dtype=torch.int32, device=dev)
        mode = torch.zeros(B, dtype=torch.int32, device=dev)
        tile_seq = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(tiles)
        tile_row = (torch.arange(tiles, dtype=torch.int32, device=dev) * tr).repeat(B)
        splits = K.attention_kv_splits(B * tiles * r.kv_slots, self.mp * K.PAGE_SIZE) if tr == K.TC_TILE_ROWS else 1
        self.plans = [K.AttentionPlan(self.table, q_start, q_len, self.kv[s], mode, tile_seq, tile_row, tr, {},
                                      splits) for s in range(S)]
        self.logq = torch.zeros(S, B, dtype=torch.float32, device=dev)
        self.logp = torch.zeros(S, B, dtype=torch.float32, device=dev)
        self.result = torch.zeros(S, B, 3, dtype=torch.float32, device=dev)
        self.result_host = torch.zeros(S, B, 3, dtype=torch.float32).pin_memory()
        self.backend = backend
        self.graph = None
        self.kernels_per_replay = 0
        if use_graph:
            s = torch.cuda.Stream(device=dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(2):
                    self._body()
            torch.cuda.current_stream(dev).wait_stream(s)
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            from ..ops import _ext

            before = _ext.launches()
            with torch.cuda.graph(g, stream=s):
                self._body()
            self.kernels_per_replay = _ext.launches() - before
            self.graph = g

    def _body(self):
        r = self.backend.runner
        self.ids[0].copy_(self.ids0)
        for s in range(self.S):
            logits = r.forward(StepMeta(self.ids[s], self.pos[s], self.slots[s], self.plans[s], None))
            K.sample(logits, self.inv_temp, self.uni[s], tokens=self.ids[s + 1], logq=self.logq[s],
                     logp=self.logp[s], arith=self.arith, next_uniforms=self.uni[s + 1], top_k=self.top_k,
                     top_p=self.top_p)
        self.result[:, :, 0].copy_(self.ids[1:])
        self.result[:, :, 1].copy_(self.logq)
        self.result[:, :, 2].copy_(self.logp)

    def run(self) -> np.ndarray:
        self.dev.copy_(self.host, non_blocking=True)
        self.uni[:self.S].copy_(self.uni_host, non_blocking=True)
        self.arith.copy_(self.arith_host, non_blocking=True)
        self.inv_temp.copy_(self.it_host, non_blocking=True)
        self.top_k.copy_(self.topk_host, non_blocking=True)
        self.top_p.copy_(self.topp_host, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            self.backend.stats["graph_kernel_launches"] += self.kernels_per_replay
        else:
            self._body()
        self.result_host.copy_(self.result, non_blocking=True)
        self.carry_host.copy_(self.uni[self.S], non_blocking=True)
        torch.cuda.current_stream(self.backend.runner.device).synchronize()
        return self.result_host.numpy()


class EngineBackend:
    """Batched sampling and scoring on the sm_100a runner (AutoregressiveBackend)."""

    # Sampled and re-scored log-probabilities of the same tokens come from different kernel
    # shapes (graphed decode steps against packed prefill rows) over bf16 activations; they
    # agree to about 0.02 per token (the GPU tests' bound).  Stored behaviour probabilities
    # are checked against re-scoring within (absolute, per token) of this.
    logprob_tolerance = (1e-3, 2e-2)

    def __init__(self, runner: ModelRunner, *, model_id: str | None = None, max_batch: int = 64,
                 bos_token_id: int | None = None, use_graphs: bool = True, prefix_cache_pages: int | None = None,
                 max_seq_tokens: int = 4096, prefill_tokens: int = 4096, decode_chunk: int = 16,
                 score_pack: int = 256, speculation: ActiveBatchSpeculationConfig | None = None,
                 draft_tree: RolloutTokenTree | None = None):
        if draft_tree is not None and speculation is None:
            raise ValueError("a draft tree needs an active-batch speculation config")
        self.runner = runner
        self.cache: KVCache = runner.cache
        self._model_id = model_id or f"b200:{runner.cfg.name}"
        self.max_batch = max_batch
        self.bos_token_id = bos_token_id
        self.use_graphs = use_graphs
        self.decode_chunk = decode_chunk
        self.score_pack = score_pack          # continuations scored per packed pass (bounds the KV it holds)
        self.max_pages = -(-(max_seq_tokens + decode_chunk) // PAGE) + 1
        self.prefill_tokens = min(prefill_tokens, runner.max_tokens)
        budget = prefix_cache_pages if prefix_cache_pages is not None else self.cache.num_pages // 2
        self.prefix = PrefixCache(self.cache, budget)
        self._graphs: dict[int, _DecodeGraph] = {}
        self._lock = threading.RLock()
        self.speculation = speculation
        self.draft_tree = draft_tree if draft_tree is not None else (
            RolloutTokenTree.from_config(speculation) if speculation is not None else None)
        self.stats = {"sample_calls": 0, "score_calls": 0, "sampled_sequences": 0, "generated_tokens": 0,
                      "prefill_tokens": 0, "reused_prefix_tokens": 0, "decode_steps": 0, "scored_tokens": 0,
                      "graph_kernel_launches": 0, "speculative_requests": 0, "speculative_hits": 0,
                      "draft_tokens_proposed": 0, "draft_tokens_accepted": 0, "verification_token_slots": 0}

    @property
    def model_id(self) -> str:
        return self._model_id

    @property
    def vocab_size(self) -> int:
        return self.runner.cfg.vocab_size

    def snapshot(self) -> dict:
        return dict(self.stats, prefix_cache_pages=len(self.prefix._pages))

    def observe_draft_samples(self, samples) -> None:
        """Feed finished samples (from this or another backend) to the draft tree."""
        if self.draft_tree is not None:
            self.draft_tree.observe_samples(samples)

    def observe_draft_sequences(self, sequences) -> None:
        if self.draft_tree is not None:
            for seq in sequences:
                self.draft_tree.observe(seq)

    def draft_cache_snapshot(self):
        return None if self.draft_tree is None else self.draft_tree.snapshot()

    def close(self) -> None:
        with self._lock:
            torch.cuda.synchronize(self.runner.device)
            for g in self._graphs.values():
                g.graph = None
            self._graphs.clear()
            self.prefix.clear()

    # ------------------------------------------------------------- helpers --
    def _model_prefix(self, prefix) -> tuple:
        if prefix:
            return tuple(prefix)
        if self.bos_token_id is None:
            raise ValueError("an empty prefix requires a bos_token_id")
        return (self.bos_token_id,)

    @staticmethod
    def _truncation(s: SamplingConfig | None) -> tuple[int, float]:
        """(top_k, top_p) of a policy in the sampler's per-row encoding (0 / 1 = off)."""
        if s is None:
            return 0, 1.0
        return (0 if s.top_k is None else int(s.top_k)), float(s.top_p)

    def _open(self, tokens: tuple, *, keep_last: bool) -> tuple[int, int]:
        """KV sequence holding ``tokens`` (minus the last one when ``keep_last``).

        Returns (seq, number of tokens whose KV still has to be computed).
        """
        n_kv = len(tokens) - 1 if keep_last else len(tokens)
        pages, _ = self.prefix.lookup(tokens, n_kv)
        reused = len(pages) * PAGE
        seq = self.cache.manager.adopt(pages, reused) if pages else self.cache.create()
        self.stats["reused_prefix_tokens"] += reused
        return seq, n_kv - reused

    def _prefill(self, items: list[tuple[int, tuple, int]]) -> None:
        """Packed prefill of the uncached tails.  items: (seq, tokens, tail_len).

        Long tails are split into ordered chunks of at most ``prefill_tokens``.
        """
        r = self.runner
        G = r.q_slots // r.kv_slots
        segments = []  # (seq, tokens, count), in causal order per sequence
        for seq, tokens, tail in items:
            while tail > 0:
                n = min(tail, self.prefill_tokens)
                segments.append((seq, tokens, n))
                tail -= n
        groups, chunk, used, seen = [], [], 0, set()
        for seg in segments:
            # a sequence appears at most once per packed forward
            if chunk and (used + seg[2] > self.prefill_tokens or seg[0] in seen):
                groups.append(chunk)
                chunk, used, seen = [], 0, set()
            chunk.append(seg)
            used += seg[2]
            seen.add(seg[0])
        if chunk:
            groups.append(chunk)
        for grp in groups:
            ids, pos, slots, qlens, kvlens, seqs = [], [], [], [], [], []
            for seq, tokens, n in grp:
                start = self.cache.length(seq)
                slots += self.cache.append(seq, n)
                ids += list(tokens[start:start + n])
                pos += list(range(start, start + n))
                qlens.append(n)
                kvlens.append(start + n)
                seqs.append(seq)
            table = torch.zeros(len(grp), self.max_pages, dtype=torch.int32)
            self.cache.fill_table(seqs, table)
            meta = build_meta(r.device, table, ids, pos, slots, qlens, kvlens, [0] * len(grp), G,
                              kv_heads=r.kv_slots)
            r.forward(meta, compute_logits=False)
            self.stats["prefill_tokens"] += len(ids)

    def _cache_pages(self, seq: int, tokens: tuple) -> None:
        n = min(self.cache.length(seq), len(tokens)) // PAGE
        if n <= 0:
            return
        keys = self.prefix.keys(tokens, n)
        self.prefix.insert(keys, list(self.cache.manager.pages(seq))[:n])

    def _graph(self, B: int, S: int) -> _DecodeGraph:
        b = next(x for x in BUCKETS if x >= B)
        g = self._graphs.get((b, S))
        if g is None:
            g = _DecodeGraph(self, b, S, self.use_graphs)
            self._graphs[(b, S)] = g
        return g

    # -------------------------------------------------------------- sample --
    def sample_batch(self, requests: Sequence[GenerationRequest]) -> list[SequenceSample]:
        with self._lock, trace_range("engine.sample_batch"):
            out: list[SequenceSample | None] = [None] * len(requests)
            pending = list(enumerate(requests))
            while pending:
                group, pending = pending[: self.max_batch], pending[self.max_batch:]
                for i, smp in self._sample_group(group):
                    out[i] = smp
            if self.draft_tree is not None:
                self.draft_tree.observe_samples(out)
            self.stats["sample_calls"] += 1
            self.stats["sampled_sequences"] += len(requests)
            return out  # type: ignore[return-value]

    def _sample_group(self, group):
        act: list[_Active] = []
        opened = []
        for i, req in group:
            tokens = self._model_prefix(req.prefix)
            seq, tail = self._open(tokens, keep_last=True)
            opened.append((seq, tokens, tail))
            if req.arithmetic_uniform is not None:
                # one code point for the whole sequence, rescaled on the device after every token
                uni = np.full(req.max_new_tokens, np.nan)
                carry = float(req.arithmetic_uniform)
            else:
                uni = (np.asarray(req.uniforms, dtype=np.float64) if req.uniforms is not None
                       else np.random.default_rng(req.seed).random(req.max_new_tokens))
                carry = None
            act.append(_Active(i, req, seq, tokens[-1], len(tokens) - 1, uni, [], [], [], carry=carry))
        self.cache.flush_copies()
        self._prefill(opened)
        for a, (seq, tokens, _) in zip(act, opened):
            self._cache_pages(seq, tokens)
        done: list[_Active] = []
        proposals = self._propose(act)
        if proposals:
            self._verify_drafts(act, proposals)
            still = []
            for a in act:
                (done if a.finish == "eos" or len(a.tokens) >= a.request.max_new_tokens else still).append(a)
            act = still
        while act:
            n = len(act)
            rem = min(a.request.max_new_tokens - len(a.tokens) for a in act)
            S = 1 << (min(self.decode_chunk, rem).bit_length() - 1)     # power of two <= the shortest remainder
            g = self._graph(n, S)
            B = g.B
            steps = np.arange(S, dtype=np.int64)[:, None]
            seqs = [a.seq for a in act]
            g.h_slots[:, :n] = np.asarray(self.cache.manager.append_many(seqs, S), dtype=np.int64).reshape(n, S).T
            starts = np.fromiter((a.pos for a in act), dtype=np.int64, count=n)
            g.h_ids[:n] = [a.last for a in act]
            g.h_pos[:, :n] = starts[None, :] + steps
            g.h_kv[:, :n] = starts[None, :] + 1 + steps
            uni = g.uni_host.numpy()
            for b, a in enumerate(act):
                if a.carry is not None:
                    uni[:, b] = a.carry
                else:
                    t = len(a.tokens)
                    uni[:, b] = a.uniforms[t:t + S]
            g.arith_host.numpy()[:n] = [a.carry is not None for a in act]
            g.it_host.numpy()[:n] = [1.0 / a.request.sampling.temperature for a in act]
            cuts = [self._truncation(a.request.sampling) for a in act]
            g.topk_host.numpy()[:n] = [c[0] for c in cuts]
            g.topp_host.numpy()[:n] = [c[1] for c in cuts]
            self.cache.manager.fill_table_np(seqs, g.h_table[:n])
            if n < B:
                g.h_slots[:, n:] = -1
                g.h_ids[n:] = 0
                g.h_pos[:, n:] = 0
                g.h_kv[:, n:] = 1
                g.h_table[n:] = 0
                g.uni_host[:, n:] = 0.5
                g.arith_host[n:] = 0
                g.topk_host[n:] = 0
                g.topp_host[n:] = 1.0
            res = g.run()
            self.stats["decode_steps"] += S
            # per sequence: how many of the S tokens it keeps (up to and including EOS, within budget)
            toks = res[:, :n, 0].astype(np.int64).T                       # [n, S]
            eos_ids = np.array([-1 if a.request.sampling.eos_token_id is None else a.request.sampling.eos_token_id
                                for a in act], dtype=np.int64)
            hit = toks == eos_ids[:, None]
            first_eos = np.where(hit.any(1), hit.argmax(1) + 1, S + 1)   # S + 1: no EOS among the S tokens
            room = np.array([a.request.max_new_tokens - len(a.tokens) for a in act], dtype=np.int64)
            keep = np.minimum(first_eos, np.minimum(room, S))
            logq_cols = res[:, :n, 1].T.tolist()
            logp_cols = res[:, :n, 2].T.tolist()
            tok_cols = toks.tolist()
            still = []
            for b, a in enumerate(act):
                k = int(keep[b])
                if a.carry is not None:
                    a.carry = float(g.carry_host[b])
                a.tokens.extend(tok_cols[b][:k])
                a.logq.extend(logq_cols[b][:k])
                a.logp.extend(logp_cols[b][:k])
                a.last, a.pos = tok_cols[b][k - 1], a.pos + k
                if first_eos[b] <= k:
                    a.finish = "eos"
                if k < S:
                    self.cache.truncate(a.seq, a.pos)      # drop KV of steps past the sequence's end
                if a.finish == "eos" or len(a.tokens) >= a.request.max_new_tokens:
                    done.append(a)
                else:
                    still.append(a)
            act = still
        results = []
        for a in done:
            full = self._model_prefix(a.request.prefix) + tuple(a.tokens)
            self._cache_pages(a.seq, full)
            self.cache.release(a.seq)
            req = a.request
            results.append((a.index, SequenceSample(
                tuple(req.prefix), tuple(a.tokens), tuple(a.logq), req.sampling.policy_id, self.model_id,
                req.request_id, a.finish, tuple(a.logp), BASE_POLICY)))
            self.stats["generated_tokens"] += len(a.tokens)
        return results

    # ---------------------------------------------------------- speculation --
    def _propose(self, act: list[_Active]) -> dict[int, DraftProposal]:
        """Draft continuations from the rollout tree for the rows of one call (tiered by its size)."""
        spec, tree = self.speculation, self.draft_tree
        if spec is None or tree is None or not act:
            return {}
        self.stats["speculative_requests"] += len(act)
        n = spec.draft_tokens(len(act))
        if n <= 0:
            return {}
        out = {}
        for j, a in enumerate(act):
            req = a.request
            if a.carry is not None:            # arithmetic coding: one code point, no per-token uniforms
                continue
            seed = SeedStream(req.seed).derive("stochastic-draft", req.request_id) if spec.stochastic_tree else None
            prop = tree.draft(self._model_prefix(req.prefix), min(n, req.max_new_tokens),
                              stochastic=spec.stochastic_tree, seed=seed)
            if prop.token_ids:
                out[j] = prop
        return out

    def _verify_drafts(self, act: list[_Active], proposals: dict[int, DraftProposal]) -> None:
        """Verify every proposal in packed forwards of (last fed token + draft) rows."""
        cap = min(self.prefill_tokens, self.runner.max_logit_rows)
        chunk, used = [], 0
        for j in sorted(proposals):
            need = len(proposals[j].token_ids) + 1
            if chunk and used + need > cap:
                self._verify_chunk(chunk)
                chunk, used = [], 0
            chunk.append((act[j], proposals[j]))
            used += need
        if chunk:
            self._verify_chunk(chunk)

    def _verify_chunk(self, chunk: list[tuple[_Active, DraftProposal]]) -> None:
        r = self.runner
        G = r.q_slots // r.kv_slots
        ids, pos, slots, qlens, kvlens, seqs = [], [], [], [], [], []
        inv_t, uni, top_k, top_p = [], [], [], []
        for a, p in chunk:
            n = len(p.token_ids) + 1
            slots += self.cache.append(a.seq, n)
            ids += [a.last] + [int(t) for t in p.token_ids]
            pos += list(range(a.pos, a.pos + n))
            qlens.append(n)
            kvlens.append(a.pos + n)
            seqs.append(a.seq)
            t0 = len(a.tokens)
            u = np.full(n, 0.5)
            have = a.uniforms[t0:t0 + n]
            u[:have.size] = have
            uni.append(u)
            cut = self._truncation(a.request.sampling)
            inv_t += [1.0 / a.request.sampling.temperature] * n
            top_k += [cut[0]] * n
            top_p += [cut[1]] * n
        table = torch.zeros(len(chunk), self.max_pages, dtype=torch.int32)
        self.cache.fill_table(seqs, table)
        meta = build_meta(r.device, table, ids, pos, slots, qlens, kvlens, [0] * len(chunk), G, kv_heads=r.kv_slots)
        logits = r.forward(meta)
        dev = logits.device
        it_d = torch.tensor(inv_t, dtype=torch.float32, device=dev)
        tk_d = torch.tensor(top_k, dtype=torch.int32, device=dev)
        tp_d = torch.tensor(top_p, dtype=torch.float32, device=dev)
        tok, lq, lp = K.sample(logits, it_d, torch.from_numpy(np.concatenate(uni)).to(dev), top_k=tk_d, top_p=tp_d)
        tok, lq, lp = tok.cpu().numpy(), lq.cpu().numpy(), lp.cpu().numpy()
        self.stats["verification_token_slots"] += len(ids)
        row = 0
        for a, p in chunk:
            D = len(p.token_ids)
            rows = slice(row, row + D + 1)
            drawn, logq, logp = tok[rows].tolist(), lq[rows].tolist(), lp[rows].tolist()
            if p.stochastic:
                self._stochastic_draws(a, p, logits[rows], it_d[rows], tk_d[rows], tp_d[rows], drawn, logq, logp)
            row += D + 1
            room = a.request.max_new_tokens - len(a.tokens)
            keep, accepted, eos = draft_acceptance(p.token_ids, drawn, room, a.request.sampling.eos_token_id)
            a.tokens.extend(drawn[:keep])
            a.logq.extend(logq[:keep])
            a.logp.extend(logp[:keep])
            a.last, a.pos = drawn[keep - 1], a.pos + keep
            self.cache.truncate(a.seq, a.pos)        # KV of the fed token and the accepted draft prefix
            if eos:
                a.finish = "eos"
            self.draft_tree.record_verification(proposed=min(D, room), accepted=accepted)
            self.stats["speculative_hits"] += 1
            self.stats["draft_tokens_proposed"] += min(D, room)
            self.stats["draft_tokens_accepted"] += accepted

    @staticmethod
    def _stochastic_draws(a: _Active, p: DraftProposal, logits, inv_t, top_k, top_p, drawn, logq, logp) -> None:
        """Replace the inverse-CDF draws of a stochastic draft's positions by speculative sampling.

        Position j keeps draft token d with probability min(1, p(d) / q(d)) (acceptance uniforms
        from the request's ``stochastic-draft-verification`` stream); a rejection draws from
        (p - q)+ / |(p - q)+| with the position's own uniform.  Positions after the first
        rejection are never used.  The entry after the draft keeps the sampler's ordinary draw.
        """
        D = len(p.token_ids)
        acc_u = np.random.default_rng(SeedStream(a.request.seed).derive(
            "stochastic-draft-verification", a.request.request_id)).random(D)
        policy = K.truncated_log_policy(logits[:D].float() * inv_t[:D, None], top_k[:D], top_p[:D])
        full = torch.log_softmax(logits[:D].float(), dim=-1)
        t0 = len(a.tokens)
        for j, d in enumerate(int(t) for t in p.token_ids):
            law = dict(p.token_distributions[j])
            q = law.get(d, 0.0)
            if q <= 0:
                raise RuntimeError("a drafted token has zero proposal probability")
            target = float(policy[j, d].exp())
            if acc_u[j] < min(1.0, target / q):
                tok = d
            else:
                resid = policy[j].double().exp()
                idx = torch.tensor(list(law), dtype=torch.long, device=resid.device)
                resid.index_add_(0, idx, -torch.tensor(list(law.values()), dtype=torch.float64, device=resid.device))
                resid.clamp_min_(0.0)
                total = float(resid.sum())
                if not math.isfinite(total) or total <= 0:
                    raise RuntimeError("a rejected stochastic draft has no residual mass")
                u = float(a.uniforms[t0 + j]) if t0 + j < a.uniforms.size else 0.5
                cdf = torch.cumsum(resid / total, 0)
                tok = min(int((cdf < u).sum()), resid.numel() - 1)
            drawn[j], logq[j], logp[j] = tok, float(policy[j, tok]), float(full[j, tok])
            if tok != d:
                return

    # --------------------------------------------------------------- score --
    def score_batch(self, requests: Sequence[ScoreRequest]) -> list[tuple[float, ...]]:
        """Per-token log-probabilities of every continuation (policy ``sampling`` or T = 1)."""
        with self._lock, trace_range("engine.score_batch"):
            flat = []
            for req in requests:
                for cont in req.continuations:
                    flat.append((self._model_prefix(req.prefix), tuple(cont), req.sampling))
            out: list = [None] * len(flat)
            packed = [i for i, (_, c, s) in enumerate(flat)
                      if c and self.runner.comm.world == 1 and self._truncation(s) == (0, 1.0)]
            for lo in range(0, len(packed), self.score_pack):
                chunk = packed[lo:lo + self.score_pack]
                for i, values in zip(chunk, self._score_packed([flat[i] for i in chunk])):
                    out[i] = values
            for i, (p, c, s) in enumerate(flat):
                if out[i] is None:
                    out[i] = self._score_one(p, c, s)
            self.stats["score_calls"] += 1
            return out

    def _score_packed(self, work: list[tuple]) -> list[tuple[float, ...]]:
        """Score many (prefix, continuation, full-support policy) items in packed forwards.

        Every item reuses the cached full pages of its prefix, its remaining tokens
        are prefilled together with the other items' (at most ``prefill_tokens`` per
        forward, a sequence at most once per forward), and the scored rows go
        through the fused head-statistics GEMM, so no logits row is stored.
        """
        r = self.runner
        G = r.q_slots // r.kv_slots
        values = [np.empty(len(c), dtype=np.float64) for _, c, _ in work]
        segments, opened = [], []
        for i, (prefix, cont, pol) in enumerate(work):
            full = prefix + cont
            first_row = len(prefix) - 1                  # position whose logits score cont[0]
            pages, _ = self.prefix.lookup(full, first_row)
            reused = len(pages) * PAGE
            seq = self.cache.manager.adopt(pages, reused) if pages else self.cache.create()
            self.stats["reused_prefix_tokens"] += reused
            opened.append((seq, full))
            inv = 1.0 if pol is None else 1.0 / pol.temperature
            pos = reused
            while pos < len(full) - 1:
                n = min(len(full) - 1 - pos, self.prefill_tokens)
                segments.append((i, seq, full, pos, n, first_row, inv))
                pos += n
        self.cache.flush_copies()
        groups, chunk, used, seen = [], [], 0, set()
        for seg in segments:
            if chunk and (used + seg[4] > self.prefill_tokens or seg[1] in seen):
                groups.append(chunk)
                chunk, used, seen = [], 0, set()
            chunk.append(seg)
            used += seg[4]
            seen.add(seg[1])
        if chunk:
            groups.append(chunk)
        for grp in groups:
            ids, pos, slots, rows, targets, inv_t = [], [], [], [], [], []
            qlens, kvlens, seqs, spans = [], [], [], []
            offset = 0
            for i, seq, full, start, n, first_row, inv in grp:
                arr = np.asarray(full, dtype=np.int64)
                slots.append(np.asarray(self.cache.append(seq, n), dtype=np.int64))
                ids.append(arr[start:start + n])
                pos.append(np.arange(start, start + n))
                qlens.append(n)
                kvlens.append(start + n)
                seqs.append(seq)
                lo = max(first_row, start)
                if lo < start + n:
                    # positions lo .. start+n-1 predict tokens lo+1 .. start+n of the continuation
                    rows.append(np.arange(lo - start, n) + offset)
                    targets.append(arr[lo + 1:start + n + 1])
                    inv_t.append(np.full(start + n - lo, inv, dtype=np.float32))
                    spans.append((i, lo - first_row, start + n - lo))
                offset += n
            table = torch.zeros(len(grp), self.max_pages, dtype=torch.int32)
            self.cache.fill_table(seqs, table)
            cat = np.concatenate
            meta = build_meta(r.device, table, cat(ids), cat(pos), cat(slots), qlens, kvlens, [0] * len(grp), G,
                              logit_rows=cat(rows) if rows else None, kv_heads=r.kv_slots)
            self.stats["prefill_tokens"] += offset
            if not rows:
                r.forward(meta, compute_logits=False)
                continue
            it = torch.from_numpy(cat(inv_t)).to(r.device, non_blocking=True)
            tg = torch.from_numpy(cat(targets).astype(np.int32)).to(r.device, non_blocking=True)
            _, _, _, logq = r.forward_stats(meta, it, tg)
            got = logq.cpu().numpy()
            at = 0
            for i, k0, count in spans:
                values[i][k0:k0 + count] = got[at:at + count]
                at += count
            self.stats["scored_tokens"] += at
        for seq, full in opened:
            self._cache_pages(seq, full)
            self.cache.release(seq)
        return [tuple(v.tolist()) for v in values]

    def score_statistics_batch(self, requests: Sequence[ScoreRequest], *, confidence_top_k: int | None = None
                               ) -> list[SequenceScoreStatistics]:
        """Per continuation: token log-probabilities plus entropy / self-certainty / top-K confidence.

        Entropy and self-certainty need finite log-probabilities over the whole
        vocabulary, so only full-support temperature policies are accepted.
        One fused kernel pass per logits row computes all statistics.
        """
        if confidence_top_k is not None and not 0 < confidence_top_k <= 16:
            raise ValueError("confidence_top_k must lie in [1, 16]")
        out = []
        with self._lock:
            for req in requests:
                pol = req.sampling or SamplingConfig()
                if not pol.full_support:
                    raise ValueError("entropy and self-certainty require a full-support policy")
                for cont in req.continuations:
                    if not cont:
                        raise ValueError("confidence rewards require nonempty continuations")
                    rows = self._score_one(self._model_prefix(req.prefix), tuple(cont), pol,
                                           stats_topk=confidence_top_k or 0)
                    V = self.runner.cfg.vocab_size
                    logp = tuple(r[0] for r in rows)
                    n = len(rows)
                    out.append(SequenceScoreStatistics(
                        logp, sum(logp) / n, sum(r[1] for r in rows) / n,
                        sum(-(math.log(V) + r[2]) for r in rows) / n,
                        tuple(r[3] for r in rows) if confidence_top_k else (), confidence_top_k))
            self.stats["score_calls"] += 1
        return out

    def next_token_probabilities(self, prefix: Sequence[int], block: Sequence[int] = ()) -> np.ndarray:
        """Temperature-1 next-token distributions after ``prefix + block[:i]`` for i = 0..len(block).

        One forward over the uncached part of ``prefix + block`` (the prefix
        cache supplies the rest); returns float64 [len(block) + 1, V] on the host.
        """
        with self._lock:
            rows: list[torch.Tensor] = []
            self._score_one(self._model_prefix(tuple(prefix)), tuple(block), None, logits_out=rows)
            logits = torch.cat(rows).double()
            return torch.softmax(logits, dim=-1).numpy()

    def _score_one(self, prefix: tuple, cont: tuple, sampling: SamplingConfig | None,
                   stats_topk: int | None = None, logits_out: list | None = None) -> tuple:
        """Per-token log-probabilities of ``cont`` (or, with ``stats_topk``, per-token statistics rows).

        With ``logits_out`` the fp32 logits rows of every position from the last
        prefix token to the last token of ``cont`` (len(cont) + 1 rows) are
        appended to it (on the host) instead.
        """
        if not cont and logits_out is None:
            return ()
        r = self.runner
        G = r.q_slots // r.kv_slots
        full = prefix + cont
        seq, _ = self._open(full, keep_last=True)
        self.cache.flush_copies()
        start = self.cache.length(seq)
        first_row = len(prefix) - 1        # position whose logits score cont[0]
        values: list[float] = []
        it = torch.full((1,), 1.0 if sampling is None else 1.0 / sampling.temperature, device=r.device)
        k_row, p_row = self._truncation(sampling)
        truncated = k_row > 0 or p_row < 1.0
        # positions [start, len(full) - 1) still need KV; logits are needed for [first_row, len(full) - 1)
        if start > first_row:
            # the cached prefix already covers scored positions: recompute from the first scored row
            self.cache.release(seq)
            pages, _ = self.prefix.lookup(full, first_row)
            seq = self.cache.manager.adopt(pages, len(pages) * PAGE) if pages else self.cache.create()
            start = self.cache.length(seq)
        end = len(full) - 1 + (1 if logits_out is not None else 0)
        pos0 = start
        while pos0 < end:
            n = min(end - pos0, r.max_logit_rows, self.prefill_tokens)
            slots = self.cache.append(seq, n)
            table = torch.zeros(1, self.max_pages, dtype=torch.int32)
            self.cache.fill_table([seq], table)
            lo = max(first_row, pos0)
            rows = list(range(lo - pos0, n))
            meta = build_meta(r.device, table, list(full[pos0:pos0 + n]), list(range(pos0, pos0 + n)), slots, [n],
                              [pos0 + n], [0], G, logit_rows=rows if rows else None, kv_heads=r.kv_slots)
            if rows and logits_out is not None:
                logits_out.append(r.forward(meta).float().cpu())
            elif rows:
                logits = r.forward(meta)
                targets = torch.tensor([full[p + 1] for p in range(lo, pos0 + n)], dtype=torch.int32,
                                       device=r.device)
                itr = it.expand(len(rows)).contiguous()
                if stats_topk is not None:
                    values += [tuple(v) for v in K.score_stats(logits, itr, targets, stats_topk).tolist()]
                else:
                    cut = {}
                    if truncated:
                        cut = {"top_k": torch.full((len(rows),), k_row, dtype=torch.int32, device=r.device),
                               "top_p": torch.full((len(rows),), p_row, dtype=torch.float32, device=r.device)}
                    _, _, logp, logq = K.row_stats(logits, itr, targets, **cut)
                    values += (logp if sampling is None else logq).tolist()
            else:
                r.forward(meta, compute_logits=False)
            self.stats["prefill_tokens"] += n
            pos0 += n
        self._cache_pages(seq, full)
        self.cache.release(seq)
        self.stats["scored_tokens"] += len(values)
        return tuple(values)
