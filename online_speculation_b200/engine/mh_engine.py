"""Asynchronous suffix-MH over a paged, prefix-shared KV cache with block speculation.

Every chain always owns one *job*: its initial extension to the full length
L, or an MH proposal that regenerates the suffix after a uniformly drawn cut.
A proposal forks the chain's KV sequence at the cut (full pages shared by
reference, the boundary page copied), so the retained prefix is never
recomputed.  All active jobs advance together, one speculative round at a
time:

    draft   : the 1-layer block-bidirectional draft head proposes K-1 tokens
              after each job's anchor (Gumbel-max at the proposal temperature);
    verify  : the target runs the causal block [anchor, candidates];
    correct : exact p/q correction keeps the accepted prefix and draws the
              first rejected position from the positive residual, so every
              emitted token follows the proposal policy exactly, and returns
              its log q (temperature 1/alpha) and log p (temperature 1).

When a job finishes it is accepted or rejected with the full Hastings ratio
(target p^alpha), and the chain starts its next update immediately: chains do
not wait for each other, so the batch stays full.  Random streams are derived
from a :class:`SeedStream` with the reference's names (("mh", chain, 0, step,
"cut" | "proposal" | "accept")), so results do not depend on scheduling.

Reference algorithm: src/inference_scaling/arllm/algorithms/mh.py:471-619
(lock-step batched chains, one backend call per update); speculation:
online-speculation/src/blockspec/parallel/generation.py:120-212.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field

import numpy as np
import torch
import torch.distributed as dist

from ..ops import kernels as K
from ..shared.mh import decide_metropolis_hastings
from ..shared.rng import SeedStream
from ..utils.tracing import trace_range
from .draft import DraftHead, FeedbackRound, SuffixLearner
from .kv_cache import KVCache
from .runner import ModelRunner, StepMeta

BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 96, 128, 192, 256)


@dataclass
class Job:
    chain: int
    kind: str                 # "extend" or "proposal"
    step: int
    cut: int
    seq: int                  # KV sequence id
    anchor: int               # token whose KV is not yet written
    n: int                    # position of the anchor == KV length
    need: int                 # tokens to generate
    seed: int
    rounds: int = 0
    tokens: list = field(default_factory=list)
    logq: list = field(default_factory=list)
    logp: list = field(default_factory=list)


@dataclass
class Chain:
    prompt: list
    tokens: list = field(default_factory=list)
    logq: list = field(default_factory=list)
    logp: list = field(default_factory=list)
    seq: int = -1
    updates_done: int = 0
    accepted: int = 0
    quota: int = 0


class _RoundGraph:
    """Static buffers (and optionally a captured CUDA graph) for one round of B blocks."""

    def __init__(self, engine: "MHEngine", B: int, use_graph: bool, Kb: int):
        self.e = engine
        self.B = B
        self.Kb = Kb
        dev = engine.device
        mp = engine.max_pages
        self.mp = mp
        # int32 metadata packed for one H2D copy: positions, slots, kv_len, table, anchors, streams
        self.n_pos = B * Kb
        self.layout = [("positions", B * Kb), ("slots", B * Kb), ("kv_len", B), ("table", B * mp),
                       ("anchors", B), ("streams", B), ("active", B)]
        total = sum(n for _, n in self.layout)
        self.host = torch.zeros(total, dtype=torch.int32).pin_memory()
        self.dev = torch.zeros(total, dtype=torch.int32, device=dev)
        self.views, off = {}, 0
        for name, n in self.layout:
            self.views[name] = self.dev[off:off + n]
            off += n
        self.host_views, off = {}, 0
        host_np = self.host.numpy()
        for name, n in self.layout:
            self.host_views[name] = host_np[off:off + n]
            off += n
        self.seeds_np = None
        self.seeds_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.seeds_np = self.seeds_host.numpy()
        self.seeds = torch.zeros(B, dtype=torch.int64, device=dev)
        self.active = torch.zeros(B, dtype=torch.float32, device=dev)
        self.stats = {"inv_target": torch.full((B * Kb,), engine.inv_temp, dtype=torch.float32, device=dev),
                      "inv_draft": torch.full((B * (Kb - 1),), engine.inv_temp, dtype=torch.float32, device=dev),
                      "lse1_t": torch.zeros(B * Kb, dtype=torch.float32, device=dev),
                      "lseT_t": torch.zeros(B * Kb, dtype=torch.float32, device=dev),
                      "lse1_d": torch.zeros(B * (Kb - 1), dtype=torch.float32, device=dev),
                      "lseT_d": torch.zeros(B * (Kb - 1), dtype=torch.float32, device=dev)}
        table = self.views["table"].view(B, mp)
        ql = [Kb] * B
        mk = lambda v: torch.full((B,), v, dtype=torch.int32, device=dev)
        starts = torch.arange(0, B * Kb, Kb, dtype=torch.int32, device=dev)
        G = engine.runner.q_slots // engine.runner.kv_slots
        # the graph is captured once, so kernel and key split are chosen for the longest sequence
        ctas = B * engine.runner.kv_slots
        tr = K.attention_tile_rows(Kb * G, ctas, mp * K.PAGE_SIZE)
        tiles_per = -(-(Kb * G) // tr)
        tile_seq = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(tiles_per)
        tile_row0 = (torch.arange(tiles_per, dtype=torch.int32, device=dev) * tr).repeat(B)
        kv_len = self.views["kv_len"]
        splits = K.attention_kv_splits(ctas * tiles_per, mp * K.PAGE_SIZE) if tr == K.TC_TILE_ROWS else 1
        self.plan_draft = K.AttentionPlan(table, starts, mk(Kb), kv_len, mk(1), tile_seq, tile_row0, tr, {}, splits)
        self.plan_verify = K.AttentionPlan(table, starts, mk(Kb), kv_len, mk(0), tile_seq, tile_row0, tr, {}, splits)
        keys = engine.shared_prefix_keys
        if keys and tr in (16, 32):
            # the prompt pages are the same pages for every job: one pass over them for all jobs
            for plan in (self.plan_draft, self.plan_verify):
                plan.shared = K.shared_prefix(table, B * Kb, keys, B, G, engine.runner.q_slots, dev)
        mask_id = engine.head.mask_token_id if engine.head is not None else 0
        self.ids_draft = torch.full((B, Kb), mask_id, dtype=torch.int32, device=dev)
        self.ids_verify = torch.zeros(B, Kb, dtype=torch.int32, device=dev)
        rows = torch.arange(B * Kb, device=dev).view(B, Kb)[:, : Kb - 1].reshape(-1)
        self.draft_rows = rows.to(torch.int64)
        self.inv_temp_rows = torch.full((B * (Kb - 1),), engine.inv_temp, dtype=torch.float32, device=dev)
        self.inv_temp = torch.full((B,), engine.inv_temp, dtype=torch.float32, device=dev)
        self.seed_index = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(Kb - 1)
        self.row_in_seq = torch.arange(Kb - 1, dtype=torch.int32, device=dev).repeat(B)
        self.row_streams = torch.zeros(B * (Kb - 1), dtype=torch.int32, device=dev)
        self.cand = torch.zeros(B * (Kb - 1), dtype=torch.int32, device=dev)
        self.out = {
            "count": torch.zeros(B, dtype=torch.int32, device=dev),
            "tail": torch.zeros(B, dtype=torch.int32, device=dev),
            "valid": torch.zeros(B, dtype=torch.int32, device=dev),
            "emitted": torch.zeros(B, Kb, dtype=torch.int32, device=dev),
            "logq": torch.zeros(B, Kb, dtype=torch.float32, device=dev),
            "logp": torch.zeros(B, Kb, dtype=torch.float32, device=dev),
        }
        # packed result for one D2H copy
        self.result = torch.zeros(B, 2 + 3 * Kb, dtype=torch.float32, device=dev)
        self.result_host = torch.zeros(B, 2 + 3 * Kb, dtype=torch.float32).pin_memory()
        self.graph = None
        self.runs = 0                     # rounds run on these buffers (the first one includes capture)
        self.teacher = None
        self.launches_per_round = 0
        if use_graph:
            self._capture()

    def _body(self):
        e, B, Kb = self.e, self.B, self.Kb
        v = self.views
        self.ids_draft[:, 0].copy_(v["anchors"])
        self.active.copy_(v["active"])
        self.row_streams.copy_(v["streams"].repeat_interleave(Kb - 1))
        meta_d = StepMeta(self.ids_draft.view(-1), v["positions"], v["slots"], self.plan_draft, self.draft_rows)
        # Under tensor parallelism both samplers work on this rank's vocabulary shard and
        # exchange per-row scalars; full logits rows are never gathered.
        shard = e.runner.vocab_shard
        dl = e.head.forward(meta_d, self.draft_rows, gather=False)
        draft_logits = e.runner._buf("draft_logits_keep", tuple(dl.shape), torch.float32)
        draft_logits.copy_(dl)
        K.gumbel_sample(draft_logits, self.inv_temp_rows, self.seeds, seed_index=self.seed_index,
                        streams=self.row_streams, row_in_seq=self.row_in_seq, salt=0x1234, tokens=self.cand,
                        shard=shard)
        self.ids_verify[:, 0].copy_(v["anchors"])
        self.ids_verify[:, 1:].copy_(self.cand.view(B, Kb - 1))
        meta_v = StepMeta(self.ids_verify.view(-1), v["positions"], v["slots"], self.plan_verify, None)
        tl = e.runner.forward(meta_v, gather=False)
        self.teacher = e.runner.last_local_logits
        K.spec_verify(tl, draft_logits, self.cand.view(B, Kb - 1), self.inv_temp, self.seeds, streams=v["streams"],
                      salt=0x777, out=self.out, stats=self.stats, shard=shard)
        o = self.out
        self.result[:, 0].copy_(o["count"])
        self.result[:, 1].copy_(o["valid"])
        self.result[:, 2:2 + Kb].copy_(o["emitted"])
        self.result[:, 2 + Kb:2 + 2 * Kb].copy_(o["logq"])
        self.result[:, 2 + 2 * Kb:].copy_(o["logp"])

    def _capture(self):
        from ..ops import _ext

        s = torch.cuda.Stream(device=self.e.device)
        s.wait_stream(torch.cuda.current_stream(self.e.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                before = _ext.launches()
                self._body()
                self.launches_per_round = _ext.launches() - before
        torch.cuda.current_stream(self.e.device).wait_stream(s)
        torch.cuda.synchronize(self.e.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._body()
        self.graph = g

    def run(self):
        self.runs += 1
        self.e.stats["h2d_bytes"] += self.host.numel() * 4 + self.seeds_host.numel() * 8
        self.e.stats["d2h_bytes"] += self.result_host.numel() * 4
        self.dev.copy_(self.host, non_blocking=True)
        self.seeds.copy_(self.seeds_host, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            self.e.stats["graph_kernel_launches"] += self.launches_per_round
        else:
            self._body()
        self.result_host.copy_(self.result, non_blocking=True)
        torch.cuda.current_stream(self.e.device).synchronize()
        return self.result_host


class _PlainGraph:
    """Static buffers (and optionally a captured CUDA graph) of S chained plain decode steps for B jobs.

    Step s decodes one token per job from the target at the proposal temperature:
    its input ids are row s of ``ids`` and the drawn tokens land in row s + 1, so a
    replay decodes S tokens per job with one host round trip.  Positions, KV slots,
    KV lengths and the random streams of all S steps are uploaded before the replay.
    """

    def __init__(self, engine: "MHEngine", B: int, S: int, use_graph: bool):
        self.e = engine
        self.B, self.S = B, S
        dev = engine.device
        r = engine.runner
        mp = engine.max_pages
        self.mp = mp
        self.layout = [("positions", S * B), ("slots", S * B), ("kv_len", S * B), ("streams", S * B),
                       ("table", B * mp), ("anchors", B)]
        total = sum(n for _, n in self.layout)
        self.host = torch.zeros(total, dtype=torch.int32).pin_memory()
        self.dev = torch.zeros(total, dtype=torch.int32, device=dev)
        self.views, self.host_views, off = {}, {}, 0
        host_np = self.host.numpy()
        for name, n in self.layout:
            self.views[name] = self.dev[off:off + n]
            self.host_views[name] = host_np[off:off + n]
            off += n
        for name in ("positions", "slots", "kv_len", "streams"):
            self.views[name] = self.views[name].view(S, B)
            self.host_views[name] = self.host_views[name].reshape(S, B)
        self.seeds_host = torch.zeros(B, dtype=torch.int64).pin_memory()
        self.seeds_np = self.seeds_host.numpy()
        self.seeds = torch.zeros(B, dtype=torch.int64, device=dev)
        self.inv_temp = torch.full((B,), engine.inv_temp, dtype=torch.float32, device=dev)
        self.ids = torch.zeros(S + 1, B, dtype=torch.int32, device=dev)
        self.logq = torch.zeros(S, B, dtype=torch.float32, device=dev)
        self.logp = torch.zeros(S, B, dtype=torch.float32, device=dev)
        table = self.views["table"].view(B, mp)
        G = r.q_slots // r.kv_slots
        tr = K.attention_tile_rows(G, B * r.kv_slots, mp * K.PAGE_SIZE)
        tiles = -(-G // tr)
        q_start = torch.arange(B, dtype=torch.int32, device=dev)
        q_len = torch.ones(B, dtype=torch.int32, device=dev)
        mode = torch.zeros(B, dtype=torch.int32, device=dev)
        tile_seq = torch.arange(B, dtype=torch.int32, device=dev).repeat_interleave(tiles)
        tile_row = (torch.arange(tiles, dtype=torch.int32, device=dev) * tr).repeat(B)
        splits = K.attention_kv_splits(B * tiles * r.kv_slots, mp * K.PAGE_SIZE) if tr == K.TC_TILE_ROWS else 1
        self.plans = [K.AttentionPlan(table, q_start, q_len, self.views["kv_len"][s], mode, tile_seq, tile_row, tr,
                                      {}, splits) for s in range(S)]
        keys = engine.shared_prefix_keys
        if keys and tr in (16, 32):
            shared = K.shared_prefix(table, B, keys, B, G, r.q_slots, dev)
            for plan in self.plans:
                plan.shared = shared
        # packed result [B, 2 + 3 S] for one D2H copy: (S - 1, valid, tokens, log q, log p)
        self.result = torch.zeros(B, 2 + 3 * S, dtype=torch.float32, device=dev)
        self.result[:, 0] = S - 1
        self.result[:, 1] = 1
        self.result_host = torch.zeros(B, 2 + 3 * S, dtype=torch.float32).pin_memory()
        self.graph = None
        self.runs = 0
        self.launches_per_round = 0
        if use_graph:
            self._capture()

    def _body(self):
        e, S = self.e, self.S
        v = self.views
        self.ids[0].copy_(v["anchors"])
        shard = e.runner.vocab_shard
        for s in range(S):
            meta = StepMeta(self.ids[s], v["positions"][s], v["slots"][s], self.plans[s], None)
            if shard is None:
                logits = e.runner.forward(meta)
                K.gumbel_sample(logits, self.inv_temp, self.seeds, streams=v["streams"][s], salt=0x777,
                                tokens=self.ids[s + 1])
                _, _, lp, lq = K.row_stats(logits, self.inv_temp, self.ids[s + 1])
                self.logq[s].copy_(lq)
                self.logp[s].copy_(lp)
                continue
            # vocabulary-parallel: local-shard draw (global noise keys), exchanged row scalars only
            local = e.runner.forward(meta, gather=False)
            tok = self.ids[s + 1]
            K.gumbel_sample(local, self.inv_temp, self.seeds, streams=v["streams"][s], salt=0x777, tokens=tok,
                            shard=shard)
            lse1, lseT, _, _ = K.row_stats(local, self.inv_temp)
            lse = shard.logsumexp(torch.stack((lse1, lseT)))
            col = tok.long() - shard.v_lo
            own = (col >= 0) & (col < shard.width)
            logit = shard.buf("plain_token_logit", (self.B,), torch.float32, local.device)
            logit.copy_(torch.where(own, local.gather(1, col.clamp(0, shard.width - 1)[:, None]).squeeze(1), 0.0))
            shard.all_reduce(logit)
            self.logq[s].copy_(logit * self.inv_temp - lse[1])
            self.logp[s].copy_(logit - lse[0])
        self.result[:, 2:2 + S].copy_(self.ids[1:].t())
        self.result[:, 2 + S:2 + 2 * S].copy_(self.logq.t())
        self.result[:, 2 + 2 * S:].copy_(self.logp.t())

    _capture = _RoundGraph._capture

    def run(self):
        self.runs += 1
        self.e.stats["h2d_bytes"] += self.host.numel() * 4 + self.seeds_host.numel() * 8
        self.e.stats["d2h_bytes"] += self.result_host.numel() * 4
        self.dev.copy_(self.host, non_blocking=True)
        self.seeds.copy_(self.seeds_host, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
            self.e.stats["graph_kernel_launches"] += self.launches_per_round
        else:
            self._body()
        self.result_host.copy_(self.result, non_blocking=True)
        torch.cuda.current_stream(self.e.device).synchronize()
        return self.result_host


class MHEngine:
    """Suffix-MH chains with speculative block drafting on one TP group."""

    def __init__(self, runner: ModelRunner, head: DraftHead | None, *, alpha: float = 4.0, length: int = 512,
                 root_seed: int = 0, learner: SuffixLearner | None = None, use_graphs: bool = True,
                 max_pages_per_seq: int | None = None, spec_policy: str = "adaptive", probe_every: int = 8,
                 plain_steps: int = 4, share_prefix: bool = False):
        self.runner = runner
        self.head = head
        self.cache: KVCache = runner.cache
        self.block = head.block_size if head is not None else 1     # no draft head: plain decoding
        self.alpha = float(alpha)
        self.inv_temp = self.alpha  # proposal temperature 1 / alpha
        self.length = int(length)
        self.seeds = SeedStream(root_seed)
        self.learner = learner
        self.use_graphs = use_graphs
        self.device = runner.device
        self.max_pages = max_pages_per_seq or 64
        self.chains: list[Chain] = []
        self.jobs: dict[int, Job] = {}
        self._graphs: dict[tuple[int, int], _RoundGraph] = {}
        if spec_policy not in ("adaptive", "always", "never"):
            raise ValueError("spec_policy is adaptive, always or never")
        self.spec_policy = spec_policy if head is not None else "never"
        self.probe_every = probe_every
        if plain_steps < 1:
            raise ValueError("plain_steps must be positive")
        self.share_prefix = share_prefix          # two-pass attention over the common prompt pages
        self.shared_prefix_keys = 0
        self.plain_steps = plain_steps    # chained decode steps per plain round
        # per-round wall time (EMA) of speculative and plain rounds and the mean emitted tokens per
        # speculative block; the adaptive policy compares expected tokens per second of the two
        self._t_spec = self._t_plain = None
        self._accept_ema = None
        self._since_spec = 0
        self.stats = {"rounds": 0, "blocks": 0, "emitted": 0, "generated": 0, "mh_updates": 0, "mh_accepted": 0,
                      "learner_updates": 0, "graph_kernel_launches": 0, "h2d_bytes": 0, "d2h_bytes": 0,
                      "spec_rounds": 0, "plain_rounds": 0}

    # ---- setup ----
    def add_chains(self, prompts: list[list[int]]) -> None:
        P = len(prompts[0])
        if any(len(p) != P for p in prompts):
            raise ValueError("prompts of one engine share a length")
        if self._graphs:
            raise RuntimeError("add every chain before the first round")
        # Chains with one prompt fork one prefilled sequence, so the full pages of prompt[:-1]
        # are the same cache pages for every job: attention reads them in one shared pass.
        # Shorter shared runs are not worth the extra pass.
        first = tuple(prompts[0]) if not self.chains else tuple(self.chains[0].prompt)
        same = all(tuple(p) == first for p in prompts)
        keys = (P - 1) // K.PAGE_SIZE * K.PAGE_SIZE
        self.shared_prefix_keys = keys if same and keys >= 4 * K.PAGE_SIZE and self.share_prefix else 0
        start = len(self.chains)
        for p in prompts:
            self.chains.append(Chain(list(p)))
        self._prefill(list(range(start, start + len(prompts))))

    def _prefill(self, chain_ids: list[int], chunk_tokens: int = 8192) -> None:
        """Prefill prompt[:-1] once per distinct prompt and open each chain's extension job.

        Chains with the same prompt fork one prefilled sequence, so they share
        its KV pages by reference.
        """
        from .runner import build_meta

        r = self.runner
        P = len(self.chains[chain_ids[0]].prompt)
        distinct: dict[tuple, int] = {}
        for c in chain_ids:
            distinct.setdefault(tuple(self.chains[c].prompt), c)
        prompts = list(distinct)
        per = max(1, chunk_tokens // max(1, P - 1))
        roots: dict[tuple, int] = {}
        for lo in range(0, len(prompts), per):
            group = prompts[lo:lo + per]
            seqs = [self.cache.create() for _ in group]
            if P > 1:
                slots, toks, pos = [], [], []
                for s, pr in zip(seqs, group):
                    slots += self.cache.append(s, P - 1)
                    toks += list(pr[:-1])
                    pos += list(range(P - 1))
                table = torch.zeros(len(group), self.max_pages, dtype=torch.int32)
                self.cache.fill_table(seqs, table)
                meta = build_meta(self.device, table, toks, pos, slots, [P - 1] * len(group), [P - 1] * len(group),
                                  [0] * len(group), r.q_slots // r.kv_slots, kv_heads=r.kv_slots)
                r.forward(meta, compute_logits=False)
            roots.update(zip(group, seqs))
        for c in chain_ids:
            ch = self.chains[c]
            seq = self.cache.fork(roots[tuple(ch.prompt)], P - 1)
            self.jobs[c] = Job(c, "extend", 0, 0, seq, ch.prompt[-1], P - 1, self.length,
                               self.seeds.derive("mh", c, 0, "extend"))
        for s in roots.values():
            self.cache.release(s)

    # ---- job bookkeeping ----
    def _next_job(self, c: int) -> None:
        ch = self.chains[c]
        if ch.updates_done >= ch.quota:
            return
        step = ch.updates_done
        cut = int(self.seeds.generator("mh", c, 0, step, "cut").integers(0, self.length))
        P = len(ch.prompt)
        full = ch.prompt + ch.tokens
        seq = self.cache.fork(ch.seq, P + cut - 1)
        self.jobs[c] = Job(c, "proposal", step, cut, seq, full[P + cut - 1], P + cut - 1, self.length - cut,
                           self.seeds.derive("mh", c, 0, step, "proposal"))

    def _finish(self, job: Job) -> None:
        ch = self.chains[job.chain]
        P = len(ch.prompt)
        L = self.length
        self.cache.truncate(job.seq, P + L - 1)
        if job.kind == "extend":
            ch.tokens, ch.logq, ch.logp = job.tokens[:L], job.logq[:L], job.logp[:L]
            ch.seq = job.seq
        else:
            cut = job.cut
            old_p, old_q = float(sum(ch.logp[cut:L])), float(sum(ch.logq[cut:L]))
            new_p, new_q = float(sum(job.logp)), float(sum(job.logq))
            d = decide_metropolis_hastings(
                current_target_log_density=self.alpha * old_p, proposed_target_log_density=self.alpha * new_p,
                forward_proposal_log_probability=new_q, reverse_proposal_log_probability=old_q,
                uniform=float(self.seeds.generator("mh", job.chain, 0, job.step, "accept").random()))
            ch.updates_done += 1
            self.stats["mh_updates"] += 1
            if d.accepted:
                ch.accepted += 1
                self.stats["mh_accepted"] += 1
                ch.tokens[cut:L] = job.tokens
                ch.logq[cut:L] = job.logq
                ch.logp[cut:L] = job.logp
                self.cache.release(ch.seq)
                ch.seq = job.seq
            else:
                self.cache.release(job.seq)
        del self.jobs[job.chain]
        self._next_job(job.chain)

    def set_quota(self, updates_per_chain: int) -> None:
        """Allow every chain `updates_per_chain` more MH updates and open their jobs."""
        for c, ch in enumerate(self.chains):
            ch.quota = ch.updates_done + updates_per_chain
            if c not in self.jobs and ch.seq >= 0:
                self._next_job(c)

    # ---- rounds ----
    def _graph(self, B: int, Kb: int) -> _RoundGraph:
        bucket = next(b for b in BUCKETS if b >= B) if B <= BUCKETS[-1] else B
        g = self._graphs.get((bucket, Kb))
        if g is None:
            g = _RoundGraph(self, bucket, self.use_graphs, Kb)
            self._graphs[(bucket, Kb)] = g
        return g

    def _speculate_next(self) -> bool:
        """Speculation policy for the next round.

        ``always`` / ``never`` are fixed.  ``adaptive`` drafts when the expected
        tokens per second of a speculative round, (mean emitted per block) / (its
        time), beat those of a plain one, ``plain_steps`` / (its time); both times and the
        acceptance are running means of measured rounds.  While a learner is
        attached, or before both kinds have been measured, a speculative round runs
        at least every ``probe_every`` rounds, so the draft keeps learning from
        verified blocks and the acceptance estimate stays current.  The emitted
        tokens follow the proposal policy exactly in both kinds of round.
        """
        if self.spec_policy != "adaptive":
            return self.spec_policy == "always"
        if self._t_spec is None:
            return True
        if self._t_plain is None:
            return False
        if self._since_spec + 1 >= self.probe_every:
            return True
        return self._accept_ema * self._t_plain > self._t_spec * self.plain_steps

    def _plain_graph(self, B: int) -> _PlainGraph:
        bucket = next(b for b in BUCKETS if b >= B) if B <= BUCKETS[-1] else B
        key = (bucket, -self.plain_steps)
        g = self._graphs.get(key)
        if g is None:
            g = _PlainGraph(self, bucket, self.plain_steps, self.use_graphs)
            self._graphs[key] = g
        return g

    def _run_spec(self, jobs, seqs, n):
        """One speculative round: returns (packed result, block width)."""
        Kb = self.block
        g = self._graph(len(jobs), Kb)
        B, nj = g.B, len(jobs)
        hv = g.host_views
        slots = np.asarray(self.cache.manager.append_many(seqs, Kb), dtype=np.int32).reshape(nj, Kb)
        pos = hv["positions"].reshape(B, Kb)
        sl = hv["slots"].reshape(B, Kb)
        pos[:nj] = n[:, None] + np.arange(Kb)
        sl[:nj] = slots
        hv["kv_len"][:nj] = n + Kb
        hv["anchors"][:nj] = [j.anchor for j in jobs]
        hv["streams"][:nj] = [j.rounds for j in jobs]
        hv["active"][:nj] = 1
        g.seeds_np[:nj] = [j.seed & ((1 << 63) - 1) for j in jobs]
        table = hv["table"].reshape(B, g.mp)
        self.cache.manager.fill_table_np(seqs, table[:nj])
        if nj < B:  # padding rows: one visible block, no cache writes
            pos[nj:] = np.arange(Kb)
            sl[nj:] = -1
            hv["kv_len"][nj:] = Kb
            hv["anchors"][nj:] = 0
            hv["streams"][nj:] = 0
            hv["active"][nj:] = 0
            table[nj:] = 0
        res = g.run().numpy()
        if (res[:nj, 1] == 0).any():
            raise RuntimeError("speculative correction reported invalid probabilities")
        if self.learner is not None:
            fb = FeedbackRound(g.ids_draft, g.views["positions"].view(B, Kb), g.views["table"].view(B, g.mp),
                               g.teacher, g.out["count"], g.active, nj)
            if self.learner.observe(fb):
                self.stats["learner_updates"] += 1
        for j in jobs:
            j.rounds += 1
        return res, Kb, g.runs

    def _run_plain(self, jobs, seqs, n):
        """``plain_steps`` chained decode steps: returns (packed result, steps)."""
        S = self.plain_steps
        g = self._plain_graph(len(jobs))
        B, nj = g.B, len(jobs)
        hv = g.host_views
        slots = np.asarray(self.cache.manager.append_many(seqs, S), dtype=np.int32).reshape(nj, S)
        steps = np.arange(S)[:, None]
        hv["positions"][:, :nj] = n[None, :] + steps
        hv["slots"][:, :nj] = slots.T
        hv["kv_len"][:, :nj] = n[None, :] + 1 + steps
        hv["streams"][:, :nj] = np.asarray([j.rounds for j in jobs])[None, :] + steps
        hv["anchors"][:nj] = [j.anchor for j in jobs]
        g.seeds_np[:nj] = [j.seed & ((1 << 63) - 1) for j in jobs]
        table = hv["table"].reshape(B, g.mp)
        self.cache.manager.fill_table_np(seqs, table[:nj])
        if nj < B:  # padding rows: no cache writes
            hv["positions"][:, nj:] = steps
            hv["slots"][:, nj:] = -1
            hv["kv_len"][:, nj:] = 1 + steps
            hv["streams"][:, nj:] = 0
            hv["anchors"][nj:] = 0
            table[nj:] = 0
        res = g.run().numpy()
        for j in jobs:
            j.rounds += S
        return res, S, g.runs

    def round(self) -> int:
        """Advance every active job by one round (speculative or plain); returns tokens generated."""
        jobs = sorted(self.jobs.values(), key=lambda j: j.chain)
        if not jobs:
            return 0
        speculate = self._speculate_next()
        started = time.perf_counter()
        self.cache.flush_copies()
        seqs = [j.seq for j in jobs]
        nj = len(jobs)
        n = np.fromiter((j.n for j in jobs), dtype=np.int64, count=nj)
        with trace_range("mh.spec_round" if speculate else "mh.plain_round"):
            res, W, runs = self._run_spec(jobs, seqs, n) if speculate else self._run_plain(jobs, seqs, n)
        counts = res[:nj, 0].astype(np.int64)
        emitted = res[:nj, 2:2 + W].astype(np.int64)
        logq = res[:nj, 2 + W:2 + 2 * W]
        logp = res[:nj, 2 + 2 * W:2 + 3 * W]
        new_len = n + 1 + counts
        self.cache.manager.truncate_many(seqs, new_len.tolist())
        generated = 0
        finished = []
        for b, j in enumerate(jobs):
            c = int(counts[b])
            take = min(c + 1, j.need - len(j.tokens))
            j.tokens.extend(emitted[b, :take].tolist())
            j.logq.extend(logq[b, :take].tolist())
            j.logp.extend(logp[b, :take].tolist())
            generated += take
            j.anchor = int(emitted[b, c])
            j.n = int(new_len[b])
            if len(j.tokens) >= j.need:
                finished.append(j)
        self.stats["rounds"] += 1
        self.stats["generated"] += generated
        if speculate:
            self.stats["emitted"] += int((counts + 1).sum())
            self.stats["blocks"] += nj
            self.stats["spec_rounds"] += 1
        else:
            self.stats["plain_rounds"] += 1
        for j in finished:
            self._finish(j)
        self._note_round(speculate, time.perf_counter() - started, float((counts + 1).mean()), runs == 1)
        return generated

    def _note_round(self, speculate: bool, seconds: float, emitted_per_job: float, first_run: bool) -> None:
        if self.spec_policy != "adaptive" or first_run:
            return                               # a round that built (and captured) its buffers is not representative
        comm = self.runner.comm
        if comm.world > 1:
            # every rank must take the same decision: use the slowest rank's round time
            t = torch.tensor([seconds], dtype=torch.float32, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=comm.group)
            seconds = float(t.item())
        ema = lambda old, new: new if old is None else 0.8 * old + 0.2 * new
        if speculate:
            self._t_spec = ema(self._t_spec, seconds)
            self._accept_ema = ema(self._accept_ema, emitted_per_job)
            self._since_spec = 0
        else:
            self._t_plain = ema(self._t_plain, seconds)
            self._since_spec += 1

    def run_until_idle(self, max_rounds: int | None = None) -> int:
        total = 0
        rounds = 0
        while self.jobs and (max_rounds is None or rounds < max_rounds):
            total += self.round()
            rounds += 1
        return total

    def close(self) -> None:
        """Release captured CUDA graphs (they may hold collective calls) and free the KV bookkeeping.

        Call this before tearing down a process group: a graph that captured
        NCCL work keeps the communicator busy at exit otherwise.
        """
        torch.cuda.synchronize(self.device)
        for g in self._graphs.values():
            g.graph = None
        self._graphs.clear()
        if self.learner is not None:
            self.learner.close()
        torch.cuda.synchronize(self.device)

    @property
    def mean_accept_length(self) -> float:
        return self.stats["emitted"] / max(1, self.stats["blocks"])
