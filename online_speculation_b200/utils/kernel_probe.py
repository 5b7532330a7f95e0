"""Time one hot kernel in isolation (and give ``ncu`` a small, self-terminating target).

    python -m online_speculation_b200.utils.kernel_probe gemm M N K [--swiglu] [--residual]
    python -m online_speculation_b200.utils.kernel_probe grouped E M K ROWS [--swiglu]
    python -m online_speculation_b200.utils.kernel_probe moe T [--preset llada-moe-7b-a1b]
    python -m online_speculation_b200.utils.kernel_probe attention B CTX [--heads 28 --kv-heads 4 --qlen 4]
    python -m online_speculation_b200.utils.kernel_probe sample ROWS V

Each subcommand builds inputs larger than L2 where the problem allows (weights
rotate through ``--copies`` buffers so back-to-back launches read HBM), runs
``--warmup`` launches, then times ``--iters`` launches captured in a CUDA
graph with CUDA events, and prints one JSON line: microseconds per launch and
the achieved bandwidth / FLOP rate against ``MEASURED_PEAKS.json`` when the
file is present.  Under ``ncu`` use ``--iters 1 --warmup 2 --no-graph``.
"""

from __future__ import annotations

import argparse
import json
import os

import torch

from ..ops import kernels as K


def _peaks() -> dict:
    here = os.path.dirname(os.path.abspath(__file__))
    path = os.path.join(here, "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f)
    except OSError:
        return {}


def _attention_timeline(t) -> list:
    """Per traced CTA: ns from entry to set-up, and per chunk the producer issue, S issue,
    P arrival at the MMA issuer, S seen and P written by the first softmax warp."""
    rows = []
    for c in range(t.shape[0]):
        if int(t[c, 0]) == 0:
            continue
        t0 = int(t[c, 0])
        rel = lambda v: None if int(v) == 0 else int(v) - t0
        chunks = []
        for j in range(24):
            vals = [rel(t[c, base + j]) for base in (2, 26, 50, 74, 98)]
            if all(v is None for v in vals):
                break
            chunks.append(dict(zip(("tma", "s_issue", "p_at_mma", "s_seen", "p_done"), vals)))
        rows.append({"cta": c, "setup": rel(t[c, 1]), "softmax_done": rel(t[c, 122]), "exit": rel(t[c, 123]),
                     "chunks": chunks})
    return rows


def _time(body, iters: int, warmup: int, graph: bool) -> float:
    for _ in range(warmup):
        body()
    torch.cuda.synchronize()
    if graph:
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(iters):
                body()
        torch.cuda.synchronize()
        run = g.replay
    else:
        def run():
            for _ in range(iters):
                body()
    run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) * 1e3 / iters


_TRACE_SLOTS = (("entry", "setup", "first_tma", "first_stage", "last_mma", "first_acc", "unused", "exit")
                + tuple(f"chunk{c}_{w}" for c in range(8) for w in ("loaded", "done"))
                + ("cluster_staged", "cluster_synced", "cluster_reduced"))


def _gemm_timeline(body) -> dict:
    """Per-CTA stamps of one launch, in microseconds after the earliest CTA entry:
    median and max over CTAs of every slot (entry, setup, first TMA, first stage
    landed, last MMA committed, first accumulator ready, exit, then the loaded /
    finished stamps of each 32-token epilogue chunk of the last tile and the
    cluster split-K reduction stamps)."""
    ext = K._ext.require()
    buf = torch.zeros(32 * 1024, dtype=torch.int64, device="cuda")
    body()
    torch.cuda.synchronize()
    ext.gemm_set_trace(buf)
    try:
        body()
        torch.cuda.synchronize()
    finally:
        ext.gemm_set_trace(None)
    t = buf.view(1024, 32).cpu()
    t = t[t[:, 0] > 0]
    t0 = int(t[:, 0].min())
    rel = (t - t0).double() / 1e3
    rel[t == 0] = float("nan")
    res = {"ctas": int(t.shape[0])}
    for i, name in enumerate(_TRACE_SLOTS):
        col = rel[:, i]
        col = col[~col.isnan()]
        if col.numel():
            res[name] = [round(float(col.median()), 2), round(float(col.max()), 2)]
    return res


class _Rotate:
    def __init__(self, items):
        self.items, self.i = items, 0

    def next(self):
        v = self.items[self.i % len(self.items)]
        self.i += 1
        return v


def _allreduce_probe(a) -> int:
    """CUDA-event time per call of the fused reduction, max over ranks; bytes = partial rows read per rank."""
    import datetime
    import json as _json
    import os

    import torch.distributed as dist

    from ..parallel.symm import NcclCollectives, SymmetricCollectives

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", local)
    group = dist.group.WORLD
    if a.algorithm == "nccl":
        comm = NcclCollectives(group, a.hidden, a.T, dev)
    else:
        comm = SymmetricCollectives(group, a.hidden, a.T, dev, algorithm=a.algorithm)
    h = torch.randn(a.T, a.hidden, device=dev).bfloat16()
    w = torch.ones(a.hidden, device=dev).bfloat16()
    x = torch.empty_like(h)
    scratch = torch.empty_like(h)

    def call():
        part = comm.partial_buffer(a.T) if hasattr(comm, "partial_buffer") else scratch
        comm.reduce_add_norm(part, h, w, x, 1e-6)

    trace = None
    if a.trace:
        trace = torch.zeros(8, dtype=torch.int64, device=dev)
        K._ext.require().allreduce_set_trace(trace)
    for _ in range(a.warmup):
        call()
    torch.cuda.synchronize()
    iters = a.iters + (a.iters % 2)       # an even count keeps the double-buffered partials in step
    run = None
    if a.algorithm != "nccl" and not a.no_graph:
        # the fused kernels capture like any kernel: time them without host launch overhead
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(iters):
                call()
        torch.cuda.synchronize()
        run = graph.replay
        run()
        torch.cuda.synchronize()
    dist.barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    if run is not None:
        run()
    else:
        for _ in range(iters):
            call()
    t1.record()
    torch.cuda.synchronize()
    us = torch.tensor([t0.elapsed_time(t1) * 1e3 / iters], device=dev)
    dist.all_reduce(us, op=dist.ReduceOp.MAX)
    K.workspace.check_status(dev)
    stamps = None
    if trace is not None:
        K._ext.require().allreduce_set_trace(None)
        rel = (trace - trace[0]).float() / 1e3
        gathered = [torch.empty_like(rel) for _ in range(world)]
        dist.all_gather(gathered, rel)
        names = ("entry", "predecessor_done", "barrier_published", "barrier_passed", "rows_loaded", "norm_reduced",
                 "output_stored", "retired")
        stamps = [{n: round(float(v), 2) for n, v in zip(names, g.tolist())} for g in gathered]
    if rank == 0:
        peer_bytes = (world - 1) * a.T * a.hidden * 2
        print(_json.dumps({"kind": "allreduce", "world": world, "T": a.T, "hidden": a.hidden, "algorithm": a.algorithm,
                           "graph": run is not None,
                           "us_per_call_max_over_ranks": float(us), "peer_bytes_read_per_rank": peer_bytes,
                           "block0_timeline_us": stamps,
                           "peer_gbs": peer_bytes / float(us) / 1e3}))
    dist.barrier()
    del comm
    dist.destroy_process_group()
    return 0


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.utils.kernel_probe")
    sub = p.add_subparsers(dest="kind", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("M", type=int)
    g.add_argument("N", type=int)
    g.add_argument("K", type=int)
    g.add_argument("--swiglu", action="store_true")
    g.add_argument("--residual", action="store_true")
    g.add_argument("--split-mode", type=int, choices=(0, 1), default=0,
                   help="split-K across a cluster reduced through DSMEM (0) or through the global workspace (1)")
    g.add_argument("--trace", action="store_true",
                   help="also print the per-CTA timeline of one launch (globaltimer stamps, microseconds)")
    gr = sub.add_parser("grouped")
    for n in ("E", "M", "K", "rows"):
        gr.add_argument(n, type=int)
    gr.add_argument("--swiglu", action="store_true")
    mo = sub.add_parser("moe")
    mo.add_argument("T", type=int)
    mo.add_argument("--preset", default="llada-moe-7b-a1b")
    at = sub.add_parser("attention")
    at.add_argument("B", type=int)
    at.add_argument("ctx", type=int)
    at.add_argument("--heads", type=int, default=28)
    at.add_argument("--kv-heads", type=int, default=4)
    at.add_argument("--qlen", type=int, default=1, help="query tokens per sequence (a causal block at the end)")
    at.add_argument("--bidirectional", action="store_true", help="every query sees every key (diffusion / draft)")
    at.add_argument("--tile-rows", type=int, default=None,
                    help="16 / 32 / 64: the mma.sync kernels; default: the tcgen05 kernel (128-row tiles)")
    at.add_argument("--kv-splits", type=int, default=None, help="tcgen05 kernel: key splits per tile (default: auto)")
    at.add_argument("--trace", action="store_true",
                    help="tcgen05 kernel: print the per-chunk timeline of the first CTAs (one extra launch)")
    at.add_argument("--shared-prefix", type=int, default=0,
                    help="the first this many keys (whole 32-key pages) are the same pages for every sequence")
    at.add_argument("--flush-l2", action="store_true",
                    help="write 256 MB between launches (outside the timed spans), as weight streaming would")
    sa = sub.add_parser("sample")
    sa.add_argument("rows", type=int)
    sa.add_argument("V", type=int)
    sa.add_argument("--gumbel", choices=("split", "one-cta"), default=None,
                    help="time the Gumbel-max draft sampler (split rows, or one CTA per row) instead of the "
                         "inverse-CDF sampler")
    ar = sub.add_parser("allreduce", help="tensor-parallel all-reduce + residual + RMSNorm (run under "
                                          "torch.distributed.run; one process per GPU)")
    ar.add_argument("T", type=int, help="token rows")
    ar.add_argument("--hidden", type=int, default=3584)
    ar.add_argument("--algorithm", choices=("auto", "oneshot", "twoshot", "nccl"), default="auto")
    ar.add_argument("--trace", action="store_true",
                    help="one-shot: print block 0's stamps of the last call on every rank (microseconds from entry)")
    for q in (g, gr, mo, at, sa, ar):
        q.add_argument("--iters", type=int, default=20)
        q.add_argument("--warmup", type=int, default=3)
        q.add_argument("--copies", type=int, default=0, help="weight buffers to rotate through (0 = auto)")
        q.add_argument("--no-graph", action="store_true")
    a = p.parse_args(argv)
    if a.kind == "allreduce":
        return _allreduce_probe(a)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(0)
    peaks = _peaks()
    out: dict = {"kind": a.kind}
    graph = not a.no_graph

    def copies(nbytes):
        return a.copies or max(1, min(16, int(3 * 126e6 // max(1, nbytes)) + 1))

    if a.kind == "gemm":
        wb = a.M * a.K * 2
        ws = _Rotate([(torch.randn(a.M, a.K, device=dev) * 0.02).bfloat16() for _ in range(copies(wb))])
        x = torch.randn(a.N, a.K, device=dev).bfloat16()
        cols = a.M // 2 if a.swiglu else a.M
        o = torch.randn(a.N, cols, device=dev).bfloat16()

        def body():
            K.linear(x, ws.next(), swiglu=a.swiglu, residual=o if a.residual else None, out=o, split_mode=a.split_mode)
        us = _time(body, a.iters, a.warmup, graph)
        flops = 2 * a.M * a.N * a.K
        bytes_ = wb + a.N * a.K * 2 + a.N * cols * 2 * (2 if a.residual else 1)
        out.update(M=a.M, N=a.N, K=a.K, split_mode=a.split_mode, us=us, tflops=flops / us / 1e6,
                   gbs=bytes_ / us / 1e3)
        if a.trace:
            out["timeline"] = _gemm_timeline(body)
    elif a.kind == "grouped":
        E, M, Kd, R = a.E, a.M, a.K, a.rows
        w = (torch.randn(E * M, Kd, device=dev) * 0.02).bfloat16()
        x = torch.randn(R, Kd, device=dev).bfloat16()
        counts = torch.full((E,), R // E, dtype=torch.int32)
        counts[: R - int(counts.sum())] += 1
        offs = torch.cat((torch.zeros(1, dtype=torch.int32), counts.cumsum(0).int())).to(dev)
        bn = K.moe_pick_bn(R, E)
        tiles = torch.zeros((M // 128) * (-(-R // 32) + E) * 4, dtype=torch.int32, device=dev)
        total = torch.zeros(1, dtype=torch.int32, device=dev)
        ext = K._ext.require()
        ext.grouped_tiles(offs, E, M // 128, bn, tiles, total)
        o = torch.empty(R, M // 2 if a.swiglu else M, dtype=torch.bfloat16, device=dev)
        wsp, ctr, st = K.workspace.gemm_workspace(dev), K.workspace.gemm_counters(dev), K.workspace.status(dev)

        def body():
            ext.grouped_gemm(w, x, o, 1 if a.swiglu else 0, tiles, total, E, bn, wsp, ctr, st)
        us = _time(body, a.iters, a.warmup, graph)
        flops = 2 * R * M * Kd
        out.update(E=E, M=M, K=Kd, rows=R, bn=bn, us=us, tflops=flops / us / 1e6)
    elif a.kind == "moe":
        from ..models.moe import PRESETS

        c = PRESETS[a.preset]
        E, H, Fd, k = c.num_experts, c.hidden_size, c.moe_intermediate_size, c.num_experts_per_tok
        router = (torch.randn(E, H, device=dev) * 0.02).bfloat16()
        gu = (torch.randn(E * 2 * Fd, H, device=dev) * 0.02).bfloat16()
        down = (torch.randn(E * H, Fd, device=dev) * 0.02).bfloat16()
        x = torch.randn(a.T, H, device=dev).bfloat16()
        h = torch.randn(a.T, H, device=dev).bfloat16()
        buf = K.MoEBuffers(a.T, E, k, H, Fd, dev)

        def body():
            K.moe_ffn(x, h, router, gu, down, top_k=k, buffers=buf)
        us = _time(body, a.iters, a.warmup, graph)
        flops = 2 * a.T * k * 3 * H * Fd + 2 * a.T * E * H
        out.update(T=a.T, us=us, tflops=flops / us / 1e6)
    elif a.kind == "attention":
        B, ctx, hq, hkv = a.B, a.ctx, a.heads, a.kv_heads
        pps = -(-ctx // 32)
        shared = min(a.shared_prefix // 32, pps)
        own = pps - shared
        kc = torch.randn(shared + B * own, hkv, 32, 128, device=dev).bfloat16()
        vc = torch.randn_like(kc)
        table = torch.cat((torch.arange(shared, dtype=torch.int32)[None].expand(B, shared),
                           shared + torch.arange(B, dtype=torch.int32)[:, None] * own
                           + torch.arange(own, dtype=torch.int32)[None]), 1).contiguous()
        plan = K.plan_attention(table, [a.qlen] * B, [ctx] * B, [int(a.bidirectional)] * B, hq // hkv, dev,
                                tile_rows=a.tile_rows, kv_splits=a.kv_splits, kv_heads=hkv)
        q = torch.randn(B * a.qlen, hq, 128, device=dev).bfloat16()
        o = torch.empty_like(q)

        def body():
            K.attention(q, kc, vc, plan, out=o)
        if a.flush_l2:
            scrub = torch.empty(128 << 20, dtype=torch.float16, device=dev)
            spans = []
            for i in range(a.warmup + a.iters):
                scrub.fill_(float(i % 7))
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                body()
                e1.record()
                spans.append((e0, e1))
            torch.cuda.synchronize()
            us = sum(x.elapsed_time(y) for x, y in spans[a.warmup:]) * 1e3 / a.iters
            out["l2"] = "flushed before every launch"
        else:
            us = _time(body, a.iters, a.warmup, graph)
        out["shared_prefix_keys"] = shared * 32
        if a.trace and plan.tile_rows == K.TC_TILE_ROWS:
            buf = torch.zeros(1024, dtype=torch.int64, device=dev)
            ext = K._ext.require()
            ext.attention_set_trace(buf)
            body()
            torch.cuda.synchronize()
            ext.attention_set_trace(None)
            out["trace"] = _attention_timeline(buf.cpu().view(8, 128))
        bytes_ = 2 * (shared * 32 + B * (ctx - shared * 32)) * hkv * 128 * 2    # distinct K/V bytes
        # causal blocks see on average about half of a prompt-sized query range
        seen = ctx if a.bidirectional or a.qlen == 1 else ctx - (a.qlen - 1) / 2
        flops = 4 * B * a.qlen * hq * seen * 128
        out.update(B=B, ctx=ctx, qlen=a.qlen, tile_rows=plan.tile_rows, kv_splits=plan.kv_splits, us=us,
                   gbs=bytes_ / us / 1e3, tflops=flops / us / 1e6)
    else:
        logits = torch.randn(a.rows, a.V, device=dev)
        it = torch.ones(a.rows, device=dev)
        uni = torch.rand(a.rows, dtype=torch.float64, device=dev)
        seeds = torch.arange(1, a.rows + 1, dtype=torch.int64, device=dev)
        tok = torch.empty(a.rows, dtype=torch.int32, device=dev)

        def body():
            if a.gumbel == "split":
                K.gumbel_sample(logits, it, seeds, tokens=tok)
            elif a.gumbel == "one-cta":
                K._ext.require().gumbel_sample(logits, it, seeds, None, None, None, 0, tok, 0, None, None, None)
            else:
                K.sample(logits, it, uni)
        out["sampler"] = a.gumbel or "inverse-cdf"
        us = _time(body, a.iters, a.warmup, graph)
        out.update(rows=a.rows, V=a.V, us=us, gbs=a.rows * a.V * 4 / us / 1e3)
    if "gbs" in out and peaks.get("hbm_gbs"):
        out["frac_hbm_of_measured"] = out["gbs"] / peaks["hbm_gbs"]
    if "tflops" in out and peaks.get("bf16_tflops"):
        out["frac_bf16_of_measured"] = out["tflops"] / peaks["bf16_tflops"]
    print(json.dumps(out))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
