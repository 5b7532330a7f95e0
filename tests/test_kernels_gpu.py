"""Numerics of every sm_100a kernel against the plain PyTorch fp32 oracle."""

import math

import pytest
import torch

from online_speculation_b200.ops import kernels as ops
from online_speculation_b200.ops import workspace

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


@pytest.mark.parametrize(
    "M,N,K",
    [(128, 16, 64), (256, 64, 512), (4608, 64, 3584), (3584, 256, 3584), (1000, 37, 200), (512, 300, 1024),
     (2048, 1024, 1536), (152064 // 8, 64, 3584), (1004, 40, 512), (4736, 256, 512),
     # split-K over 3-, 5-, 6- and 7-CTA clusters (ragged token slices per cluster rank)
     (2304, 64, 3584), (3840, 64, 2048), (2944, 48, 4096), (2688, 40, 3584)],
)
def test_gemm_matches_fp32(cuda, M, N, K):
    torch.manual_seed(0)
    w = (torch.randn(M, K, device=cuda) * 0.05).bfloat16()
    x = torch.randn(N, K, device=cuda).bfloat16()
    out = ops.linear(x, w)
    ref = ops.linear_reference(x, w)
    torch.cuda.synchronize()
    workspace.check_status(cuda)
    assert _rel(out, ref) < 1e-2


def test_gemm_bias_residual_fp32_out(cuda):
    torch.manual_seed(1)
    M, N, Kd = 768, 48, 896
    w = (torch.randn(M, Kd, device=cuda) * 0.05).bfloat16()
    x = torch.randn(N, Kd, device=cuda).bfloat16()
    b = torch.randn(M, device=cuda).bfloat16()
    r = torch.randn(N, M, device=cuda).bfloat16()
    out = ops.linear(x, w, bias=b, residual=r)
    assert _rel(out, ops.linear_reference(x, w, bias=b, residual=r)) < 1e-2
    out32 = ops.linear(x, w, out_dtype=torch.float32)
    assert out32.dtype == torch.float32
    assert _rel(out32, ops.linear_reference(x, w)) < 1e-3
    # in-place residual stream update
    h = r.clone()
    ops.linear(x, w, residual=h, out=h)
    assert _rel(h, ops.linear_reference(x, w, residual=r)) < 1e-2


@pytest.mark.parametrize("N,split", [(64, True), (200, False), (16, True)])
def test_gemm_swiglu(cuda, N, split):
    torch.manual_seed(2)
    F, H = 320, 512
    g = (torch.randn(F, H, device=cuda) * 0.05).bfloat16()
    u = (torch.randn(F, H, device=cuda) * 0.05).bfloat16()
    w = ops.interleave_gate_up(g, u)
    x = torch.randn(N, H, device=cuda).bfloat16()
    out = ops.linear(x, w, swiglu=True, allow_split=split)
    ref = torch.nn.functional.silu(x.float() @ g.float().t()) * (x.float() @ u.float().t())
    assert _rel(out[:, :F], ref) < 1e-2


def test_gemm_repeated_split_counters_reset(cuda):
    w = (torch.randn(1024, 4096, device=cuda) * 0.02).bfloat16()
    x = torch.randn(64, 4096, device=cuda).bfloat16()
    ref = ops.linear_reference(x, w)
    for _ in range(5):
        assert _rel(ops.linear(x, w), ref) < 1e-2
    assert int(workspace.gemm_counters(cuda).abs().sum()) == 0


@pytest.mark.parametrize("M,N,K,swiglu,residual", [(3584, 256, 3584, False, True), (1024, 40, 4096, False, False),
                                                (640, 96, 2048, True, False)])
def test_gemm_workspace_split_mode(cuda, M, N, K, swiglu, residual):
    """Split-K through the global fp32 workspace (the last split to arrive reduces)."""
    torch.manual_seed(3)
    w = (torch.randn(M, K, device=cuda) * 0.05).bfloat16()
    x = torch.randn(N, K, device=cuda).bfloat16()
    r = torch.randn(N, M, device=cuda).bfloat16() if residual else None
    out = ops.linear(x, w, swiglu=swiglu, residual=r, split_mode=1)
    ref = ops.linear_reference(x, w, swiglu=swiglu, residual=r)
    torch.cuda.synchronize()
    workspace.check_status(cuda)
    assert _rel(out, ref) < 1e-2, (M, N, K)
    assert int(workspace.gemm_counters(cuda).abs().sum()) == 0


def _paged_case(device, lengths, Hkv, pages_per_seq, seed=0):
    torch.manual_seed(seed)
    B = len(lengths)
    num_pages = B * pages_per_seq + 3
    perm = torch.randperm(num_pages)[: B * pages_per_seq].view(B, pages_per_seq).int()
    k = torch.randn(num_pages, Hkv, ops.PAGE_SIZE, 128, device=device).bfloat16()
    v = torch.randn(num_pages, Hkv, ops.PAGE_SIZE, 128, device=device).bfloat16()
    return perm, k, v


ATTENTION_CASES = [
    ([1, 1, 1], [1, 33, 700], [0, 0, 0], 28, 4),       # decode
    ([4, 4], [130, 4], [0, 0], 28, 4),                 # verify block
    ([4, 4], [517, 9], [1, 1], 28, 4),                 # bidirectional draft block
    ([300, 64], [300, 64], [0, 1], 12, 2),             # prefill + diffusion
    ([1, 5], [1000, 999], [0, 1], 4, 1),               # TP-sharded heads
    ([512], [512], [0], 28, 4),                        # causal prefill over 28 row tiles of 128
    ([37, 4], [1061, 70], [0, 0], 16, 2),              # prompt chunk after history; ragged last chunk
]

# (tile_rows, kv_splits): None = the tcgen05 kernel (128-row tiles, key ranges merged in a
# cluster of kv_splits CTAs); 16 / 32 / 64 = the mma.sync kernels kept for comparison
ATTENTION_KERNELS = [(None, 1), (None, 2), (None, 4), (None, 8), (16, 1), (32, 1), (64, 1)]


@pytest.mark.parametrize("q_lens,kv_lens,modes,Hq,Hkv", ATTENTION_CASES)
@pytest.mark.parametrize("tile_rows,kv_splits", ATTENTION_KERNELS)
def test_attention_matches_fp32(cuda, q_lens, kv_lens, modes, Hq, Hkv, tile_rows, kv_splits):
    pps = max((kv + 31) // 32 for kv in kv_lens)
    table, kc, vc = _paged_case(cuda, kv_lens, Hkv, pps)
    T = sum(q_lens)
    q = torch.randn(T, Hq, 128, device=cuda).bfloat16()
    plan = ops.plan_attention(table, q_lens, kv_lens, modes, Hq // Hkv, cuda, tile_rows=tile_rows,
                              kv_splits=kv_splits)
    out = torch.full_like(q, float("nan"))
    ops.attention(q, kc, vc, plan, out=out)
    ref = ops.attention_reference(q.cpu(), kc.cpu(), vc.cpu(), plan.host, 128 ** -0.5)
    torch.cuda.synchronize()
    workspace.check_status(cuda)
    assert torch.isfinite(out).all()
    assert _rel(out.cpu(), ref) < 2e-2, (tile_rows, kv_splits)


def test_attention_default_plan_choice(cuda):
    table, kc, vc = _paged_case(cuda, [1024] * 2, 1, 32)
    plan = ops.plan_attention(table, [4, 4], [1024, 1024], [0, 0], 7, cuda, kv_heads=1)
    assert plan.tile_rows == 128 and plan.kv_splits == 8     # 2 tiles x 1 head: long key ranges are split
    plan = ops.plan_attention(table, [4] * 2, [1024] * 2, [0] * 2, 7, cuda, kv_heads=148)
    assert plan.tile_rows == 32 and plan.kv_splits == 1      # many short tiles: mma.sync key groups
    plan = ops.plan_attention(table, [300, 64], [300, 64], [0, 1], 6, cuda, kv_heads=2)
    assert plan.tile_rows == 128                             # prefill / diffusion: full tiles


@pytest.mark.parametrize("tile_rows,kv_splits", [(None, 1), (None, 4), (16, 1), (32, 1)])
def test_attention_ignores_non_finite_rows_past_the_end(cuda, tile_rows, kv_splits):
    # cache rows past a sequence's end may hold anything (recycled or never-written pages)
    kv_lens = [37, 70, 5]
    table, kc, vc = _paged_case(cuda, kv_lens, 4, 3, seed=3)
    for b, n in enumerate(kv_lens):
        for key in range(n, 96):
            page = int(table[b, key // 32])
            kc[page, :, key % 32] = float("nan")
            vc[page, :, key % 32] = float("inf")
    q_lens = [4, 4, 1]
    q = torch.randn(sum(q_lens), 28, 128, device=cuda).bfloat16()
    plan = ops.plan_attention(table, q_lens, kv_lens, [0, 1, 0], 7, cuda, tile_rows=tile_rows, kv_splits=kv_splits)
    out = ops.attention(q, kc, vc, plan)
    ref = ops.attention_reference(q.cpu(), torch.nan_to_num(kc.cpu()), torch.nan_to_num(vc.cpu()), plan.host,
                                  128 ** -0.5)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    assert _rel(out.cpu(), ref) < 2e-2


@pytest.mark.parametrize("q_len,mode,tile_rows", [(1, 0, 16), (4, 0, 16), (4, 1, 16), (4, 0, 32), (1, 0, 32)])
def test_two_pass_shared_prefix_attention_matches_one_pass(cuda, q_len, mode, tile_rows):
    """Sequences whose first pages are the same cache pages: the shared-prefix pass plus the
    per-sequence pass equal one pass over all keys (and the fp32 oracle)."""
    torch.manual_seed(q_len + mode + tile_rows)
    B, Hq, Hkv, shared_keys = 9, 28, 4, 192
    kv_lens = [shared_keys + q_len + 7 * b for b in range(B)]        # every sequence has own keys too
    own_pages = [(kv - shared_keys + 31) // 32 for kv in kv_lens]
    sp = shared_keys // 32
    kc = torch.randn(sp + sum(own_pages), Hkv, 32, 128, device=cuda).bfloat16()
    vc = torch.randn_like(kc)
    width = sp + max(own_pages)
    table = torch.zeros(B, width, dtype=torch.int32)
    nxt = sp
    for b in range(B):
        table[b, :sp] = torch.arange(sp)
        table[b, sp:sp + own_pages[b]] = torch.arange(nxt, nxt + own_pages[b])
        nxt += own_pages[b]
    q = torch.randn(B * q_len, Hq, 128, device=cuda).bfloat16()
    plan = ops.plan_attention(table, [q_len] * B, kv_lens, [mode] * B, Hq // Hkv, cuda, tile_rows=tile_rows)
    one = ops.attention(q, kc, vc, plan)
    plan.shared = ops.shared_prefix(plan.table, B * q_len, shared_keys, B, Hq // Hkv, Hq, cuda)
    two = ops.attention(q, kc, vc, plan)
    ref = ops.attention_reference(q.cpu(), kc.cpu(), vc.cpu(), plan.host, 128 ** -0.5)
    torch.cuda.synchronize()
    workspace.check_status(cuda)
    assert torch.isfinite(two).all()
    assert _rel(two.cpu(), ref) < 2e-2 and _rel(two, one) < 1e-2


def test_rmsnorm_and_fused_add(cuda):
    x = torch.randn(37, 3584, device=cuda).bfloat16()
    w = (1 + 0.1 * torch.randn(3584, device=cuda)).bfloat16()
    y = ops.rmsnorm(x, w, 1e-6)
    ref = ops.rmsnorm(x.cpu(), w.cpu(), 1e-6)
    assert _rel(y.cpu(), ref) < 1e-2
    d = torch.randn_like(x)
    h = torch.empty_like(x)
    y2 = ops.rmsnorm(x, w, 1e-6, residual=h, delta=d)
    h_ref = torch.empty_like(x.cpu())
    ref2 = ops.rmsnorm(x.cpu(), w.cpu(), 1e-6, residual=h_ref, delta=d.cpu())
    assert _rel(h.cpu(), h_ref) < 1e-2 and _rel(y2.cpu(), ref2) < 1e-2


@pytest.mark.parametrize("with_norm", [False, True])
def test_rope_cache(cuda, with_norm):
    T, Hq, Hkv = 9, 7, 2
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device=cuda).bfloat16()
    pos = torch.tensor([0, 1, 5, 100, 511, 1023, 7, 8, 9], dtype=torch.int32, device=cuda)
    slots = torch.tensor([0, 1, 2, 33, 64, 95, -1, 40, 41], dtype=torch.int32, device=cuda)
    inv = ops.rope_frequencies(128, 1e6).to(cuda)
    qn = (1 + 0.1 * torch.randn(128, device=cuda)).bfloat16() if with_norm else None
    kn = (1 + 0.1 * torch.randn(128, device=cuda)).bfloat16() if with_norm else None
    kc = torch.zeros(4, Hkv, 32, 128, device=cuda).bfloat16()
    vc = torch.zeros_like(kc)
    q = torch.empty(T, Hq, 128, device=cuda).bfloat16()
    ops.rope_cache(qkv, pos, slots, inv, q, kc, vc, Hq, Hkv, q_norm=qn, k_norm=kn)
    kc2, vc2, q2 = kc.cpu().zero_(), vc.cpu().zero_(), torch.empty_like(q.cpu())
    ops.rope_cache(qkv.cpu(), pos.cpu(), slots.cpu(), inv.cpu(), q2, kc2, vc2, Hq, Hkv,
                 q_norm=None if qn is None else qn.cpu(), k_norm=None if kn is None else kn.cpu())
    assert _rel(q.cpu(), q2) < 1e-2
    assert _rel(kc.cpu(), kc2) < 1e-2
    assert torch.equal(vc.cpu(), vc2)


def test_embed_and_page_copy(cuda):
    table = torch.randn(1000, 256, device=cuda).bfloat16()
    ids = torch.tensor([3, 999, 0, 3], dtype=torch.int32, device=cuda)
    assert torch.equal(ops.embed(ids, table), table[ids.long()])
    cache = torch.randn(3, 6, 2, 32, 128, device=cuda).bfloat16()
    ref = cache.clone()
    pairs = torch.tensor([[1, 4, 17], [2, 5, 32]], dtype=torch.int32, device=cuda)
    ops.page_copy(cache, pairs)
    ref[:, 4, :, :17] = ref[:, 1, :, :17]
    ref[:, 5] = ref[:, 2]
    assert torch.equal(cache, ref)


def test_sample_matches_float64_cdf(cuda):
    torch.manual_seed(3)
    R, V = 64, 152064
    logits = torch.randn(R, V, device=cuda) * 3
    inv_t = torch.full((R,), 4.0, device=cuda)
    inv_t[::2] = 1.0
    u = torch.rand(R, dtype=torch.float64, device=cuda)
    tok, lq, lp = ops.sample(logits, inv_t, u)
    rt, rq, rp = ops.sample_reference(logits.cpu(), inv_t.cpu(), u.cpu())
    assert (tok.cpu() == rt).float().mean() > 0.9
    # every token must sit on the float64 CDF interval containing u (up to fp32 rounding of p)
    log_q = (logits.cpu().float() * inv_t.cpu()[:, None]).log_softmax(-1)
    cdf = log_q.exp().double().cumsum(-1)
    t = tok.cpu().long()
    upper = cdf.gather(-1, t[:, None]).squeeze(-1)
    lower = torch.where(t > 0, cdf.gather(-1, (t - 1).clamp_min(0)[:, None]).squeeze(-1), torch.zeros_like(upper))
    assert bool(((lower - 1e-5 < u.cpu()) & (u.cpu() <= upper + 1e-5)).all())
    same = tok.cpu() == rt
    assert torch.allclose(lq.cpu()[same], rq[same], atol=1e-3)
    assert torch.allclose(lp.cpu()[same], rp[same], atol=1e-3)


def test_sample_edge_uniforms(cuda):
    logits = torch.randn(4, 1000, device=cuda)
    u = torch.tensor([0.0, 1e-300, 0.999999999999, 0.5], dtype=torch.float64, device=cuda)
    tok, _, _ = ops.sample(logits, None, u)
    rt, _, _ = ops.sample_reference(logits.cpu(), None, u.cpu())
    assert torch.equal(tok.cpu(), rt)


def _truncation_rows(R, V, device):
    ks = torch.tensor([0, 1, 5, 50, 1000, 0, 20, V], dtype=torch.int32).repeat(R // 8 + 1)[:R]
    ps = torch.tensor([1.0, 0.9, 1.0, 0.5, 0.95, 0.1, 0.7, 0.3], dtype=torch.float32).roll(3).repeat(R // 8 + 1)[:R]
    return ks.to(device), ps.to(device)


def test_sample_truncated_policies_match_oracle(cuda):
    torch.manual_seed(21)
    R, V = 48, 152064
    logits = torch.randn(R, V, device=cuda) * 3
    inv_t = torch.full((R,), 1.0, device=cuda)
    inv_t[1::3] = 1.25
    ks, ps = _truncation_rows(R, V, cuda)
    u = torch.rand(R, dtype=torch.float64, device=cuda)
    tok, lq, lp = ops.sample(logits, inv_t, u, top_k=ks, top_p=ps)
    log_q = ops.truncated_log_policy(logits.cpu() * inv_t.cpu()[:, None], ks.cpu(), ps.cpu())
    t = tok.cpu().long()
    assert bool(torch.isfinite(log_q.gather(-1, t[:, None])).all())          # every draw inside the kept set
    cdf = log_q.exp().double().cumsum(-1)
    upper = cdf.gather(-1, t[:, None]).squeeze(-1)
    lower = torch.where(t > 0, cdf.gather(-1, (t - 1).clamp_min(0)[:, None]).squeeze(-1), torch.zeros_like(upper))
    assert bool(((lower - 1e-5 < u.cpu()) & (u.cpu() <= upper + 1e-5)).all())
    rt, rq, rp = ops.sample_reference(logits.cpu(), inv_t.cpu(), u.cpu(), top_k=ks.cpu(), top_p=ps.cpu())
    assert (t == rt.long()).float().mean() > 0.9
    assert torch.allclose(lq.cpu(), log_q.gather(-1, t[:, None]).squeeze(-1), atol=1e-3)
    assert torch.allclose(lp.cpu(), logits.cpu().log_softmax(-1).gather(-1, t[:, None]).squeeze(-1), atol=1e-3)


def test_row_stats_truncated_policies(cuda):
    torch.manual_seed(22)
    R, V = 32, 50000
    x = torch.randn(R, V, device=cuda) * 2
    it = torch.full((R,), 2.0, device=cuda)
    ks, ps = _truncation_rows(R, V, cuda)
    log_q = ops.truncated_log_policy(x.cpu() * it.cpu()[:, None], ks.cpu(), ps.cpu())
    # half the targets inside the kept set (the argmax), half outside where the row truncates
    tg = x.argmax(-1).to(torch.int32)
    tg[1::2] = x[1::2].argmin(-1).to(torch.int32)
    lse1, lseT, logp, logq = ops.row_stats(x, it, tg, top_k=ks, top_p=ps)
    want = log_q.gather(-1, tg.cpu().long()[:, None]).squeeze(-1)
    finite = torch.isfinite(want)
    assert torch.equal(torch.isfinite(logq.cpu()), finite) and bool((~finite).any())
    assert torch.allclose(logq.cpu()[finite], want[finite], atol=1e-3)
    ref = ops.row_stats(x.cpu(), it.cpu(), tg.cpu(), top_k=ks.cpu(), top_p=ps.cpu())
    assert torch.allclose(lseT.cpu(), ref[1], atol=1e-3) and torch.allclose(lse1.cpu(), ref[0], atol=1e-3)


@pytest.mark.parametrize("rows,V", [(300, 151936), (37, 1000), (1, 129)])
def test_head_stats_match_fp32_oracle(cuda, rows, V):
    torch.manual_seed(rows + V)
    H = 1536
    x = (torch.randn(rows, H, device=cuda) * 0.5).to(torch.bfloat16)
    w = (torch.randn(V, H, device=cuda) * 0.05).to(torch.bfloat16)
    inv = torch.rand(rows, device=cuda) * 1.5 + 0.5
    tg = torch.randint(0, V, (rows,), dtype=torch.int32, device=cuda)
    tg[::5] = -1                                            # an out-of-range target scores -inf
    lse1, lseT, logp, logq = ops.head_stats(x, w, inv, tg)
    logits = x.float() @ w.float().t()
    want1 = torch.logsumexp(logits, -1)
    wantT = torch.logsumexp(logits * inv[:, None], -1)
    assert torch.allclose(lse1, want1, atol=2e-3, rtol=1e-4) and torch.allclose(lseT, wantT, atol=2e-3, rtol=1e-4)
    ok = tg >= 0
    idx = tg.clamp_min(0).long()[:, None]
    assert torch.allclose(logp[ok], (logits.gather(-1, idx).squeeze(-1) - want1)[ok], atol=2e-3, rtol=1e-4)
    assert torch.allclose(logq[ok], (logits.gather(-1, idx).squeeze(-1) * inv - wantT)[ok], atol=2e-3, rtol=1e-4)
    assert bool(torch.isinf(logp[~ok]).all()) and bool(torch.isinf(logq[~ok]).all())
    workspace.check_status()


@pytest.mark.parametrize("bl,tc,mode", [(32, 4, "prio"), (32, 32, "prio"), (256, 17, "prio"), (64, 8, "position"),
                                         (96, 5, "subset")])
def test_remask_select_matches_torch_path(cuda, bl, tc, mode):
    torch.manual_seed(bl + tc)
    B, P, mask = 6, 40, 999
    S = P + 2 * bl
    tokens = torch.randint(0, 500, (B, S), dtype=torch.int64)
    a0 = P + bl
    region = torch.rand(B, bl) < 0.6
    region[:, :tc] = True                                 # at least tc masked positions per row
    tokens[:, a0:a0 + bl] = torch.where(region, torch.full_like(region, mask, dtype=torch.int64),
                                        tokens[:, a0:a0 + bl])
    drawn = torch.randint(0, 500, (B * bl,), dtype=torch.int32)
    prio = None if mode == "position" else torch.randn(B * bl)
    logq = -torch.rand(B * bl) * 5
    traj_cpu = torch.zeros(B, dtype=torch.float64)
    traj_gpu = traj_cpu.to(cuda)
    t_cpu, t_gpu = tokens.clone(), tokens.to(cuda)
    want = ops.remask_select(t_cpu, a0, bl, mask, drawn, tc, prio=prio, logq=logq, subset=mode == "subset",
                             traj=traj_cpu, pos_offset=bl)
    got = ops.remask_select(t_gpu, a0, bl, mask, drawn.to(cuda), tc, prio=None if prio is None else prio.to(cuda),
                            logq=logq.to(cuda), subset=mode == "subset", traj=traj_gpu, pos_offset=bl)
    assert torch.equal(t_gpu.cpu(), t_cpu)
    assert torch.equal(got[0].cpu(), want[0]) and torch.equal(got[1].cpu(), want[1])
    assert torch.allclose(got[2].cpu(), want[2], atol=1e-9) and torch.allclose(traj_gpu.cpu(), traj_cpu, atol=1e-9)


def test_row_stats(cuda):
    x = torch.randn(10, 50000, device=cuda) * 2
    it = torch.full((10,), 2.0, device=cuda)
    tg = torch.randint(0, 50000, (10,), dtype=torch.int32, device=cuda)
    a = ops.row_stats(x, it, tg)
    b = ops.row_stats(x.cpu(), it.cpu(), tg.cpu())
    for u, v in zip(a, b):
        assert torch.allclose(u.cpu(), v, atol=1e-3)


def test_gumbel_sampling_distribution(cuda):
    torch.manual_seed(4)
    V, R = 16, 40000
    base = torch.randn(V) * 1.5
    logits = base.to(cuda).expand(R, V).contiguous()
    seeds = torch.tensor([12345], dtype=torch.int64, device=cuda)
    idx = torch.zeros(R, dtype=torch.int32, device=cuda)
    streams = torch.arange(R, dtype=torch.int32, device=cuda)
    inv = torch.full((R,), 0.5, device=cuda)
    tok = ops.gumbel_sample(logits, inv, seeds, seed_index=idx, streams=streams)
    freq = torch.bincount(tok.long().cpu(), minlength=V).float() / R
    p = (base * 0.5).softmax(-1)
    assert float((freq - p).abs().sum() / 2) < 0.02


def test_gumbel_split_rows_match_one_cta_per_row(cuda):
    """Few rows: the vocabulary is split over CTAs; the draw equals the one-CTA-per-row draw."""
    from online_speculation_b200.ops import _ext

    torch.manual_seed(6)
    R, V = 8, 152064
    logits = torch.randn(R, V, device=cuda) * 3
    seeds = torch.tensor([11, 12], dtype=torch.int64, device=cuda)
    si = torch.tensor([0, 1] * 4, dtype=torch.int32, device=cuda)
    streams = torch.arange(R, dtype=torch.int32, device=cuda)
    rin = torch.arange(R, dtype=torch.int32, device=cuda) % 4
    inv = torch.full((R,), 0.8, device=cuda)
    for _ in range(3):
        got = ops.gumbel_sample(logits, inv, seeds, seed_index=si, streams=streams, row_in_seq=rin, salt=5)
        want = torch.empty(R, dtype=torch.int32, device=cuda)
        _ext.require().gumbel_sample(logits, inv, seeds, si, streams, rin, 5, want, 0, None, None, None)
        assert torch.equal(got, want)
        streams += R
    best, count = workspace.sampler_split(cuda)
    torch.cuda.synchronize()
    assert int(best.abs().sum()) == 0 and int(count.abs().sum()) == 0      # the scratch is back at rest


def test_row_stats_split_rows_match_one_cta_per_row(cuda):
    """Few rows: statistics are reduced over column chunks and merged by the last CTA."""
    from online_speculation_b200.ops import _ext

    torch.manual_seed(7)
    for R, V in ((8, 152064), (100, 65536), (3, 20000)):
        logits = torch.randn(R, V, device=cuda) * 4
        inv = torch.rand(R, device=cuda) + 0.5
        tg = torch.randint(0, V, (R,), dtype=torch.int32, device=cuda)
        for _ in range(2):
            got = ops.row_stats(logits, inv, tg)
            want = [torch.empty(R, device=cuda) for _ in range(4)]
            _ext.require().row_stats(logits, inv, tg, *want, None, None, None, None)
            for g, w in zip(got, want):
                assert torch.allclose(g, w, atol=1e-4, rtol=1e-5)
        ref = torch.logsumexp(logits.double(), -1)
        assert torch.allclose(got[0].double(), ref, atol=1e-4)
    torch.cuda.synchronize()
    assert int(workspace.row_stats_split(cuda)[1].abs().sum()) == 0       # counters back at rest


def test_device_index_checks_skip_out_of_range_accesses(cuda):
    """Token ids outside the table and KV slots beyond the cache are reported, not followed.

    Each buffer is a view of a larger allocation whose extra row is a sentinel, so an
    unchecked access would stay inside this test's own memory (and show up)."""
    st = workspace.status(cuda)
    torch.cuda.synchronize()
    st.zero_()
    table_full = torch.randn(1001, 256, device=cuda).bfloat16()
    table_full[1000] = 7.0
    table = table_full[:1000]
    ids = torch.tensor([3, 1000, 5, -1], dtype=torch.int32, device=cuda)
    out = ops.embed(ids, table, torch.empty(4, 256, dtype=torch.bfloat16, device=cuda))
    torch.cuda.synchronize()
    assert torch.equal(out[0], table[3]) and torch.equal(out[2], table[5])
    assert int(out[1].abs().sum()) == 0 and int(out[3].abs().sum()) == 0
    assert int(st.item()) == 7
    st.zero_()
    Hq, Hkv, P = 4, 2, 32
    k_full = torch.zeros(5, Hkv, P, 128, dtype=torch.bfloat16, device=cuda)
    v_full = torch.zeros_like(k_full)
    kc, vc = k_full[:4], v_full[:4]                     # capacity 4 * 32 = 128 slots
    T = 3
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device=cuda).bfloat16()
    pos = torch.tensor([0, 1, 2], dtype=torch.int32, device=cuda)
    slots = torch.tensor([5, 128, 127], dtype=torch.int32, device=cuda)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, 128, 2, device=cuda).float() / 128))
    q_out = torch.empty(T, Hq, 128, dtype=torch.bfloat16, device=cuda)
    ops.rope_cache(qkv, pos, slots, inv_freq, q_out, kc, vc, Hq, Hkv)
    torch.cuda.synchronize()
    assert int(k_full[4].abs().sum()) == 0 and int(v_full[4].abs().sum()) == 0   # sentinel page untouched
    assert int(kc[0, :, 5].abs().sum()) > 0 and int(vc[3, :, 31].abs().sum()) > 0  # valid slots stored
    assert int(st.item()) == 7
    st.zero_()


def test_spec_verify_preserves_target_law(cuda):
    """Marginal law of the first emitted token must equal the target p."""
    torch.manual_seed(5)
    V, n, B = 12, 3, 30000
    tl = torch.randn(n + 1, V) * 1.5
    dl = torch.randn(n, V) * 1.5
    target = tl.to(cuda).repeat(B, 1)
    draft = dl.to(cuda).repeat(B, 1)
    inv = torch.full((B,), 1.0, device=cuda)
    q = dl.softmax(-1)
    cands = torch.stack([torch.multinomial(q[i], B, replacement=True) for i in range(n)], 1).int().to(cuda)
    seeds = torch.randint(0, 2**62, (B,), dtype=torch.int64, device=cuda)
    res = ops.spec_verify(target, draft, cands, inv, seeds)
    assert bool(res["valid"].all())
    first = res["emitted"][:, 0].long().cpu()
    freq = torch.bincount(first, minlength=V).float() / B
    p0 = tl[0].softmax(-1)
    assert float((freq - p0).abs().sum() / 2) < 0.02
    # accepted prefix length follows the min(1, p/q) acceptance of position 0
    accept0 = float((res["count"] > 0).float().mean())
    expected = float(torch.minimum(tl[0].softmax(-1), q[0]).sum())
    assert abs(accept0 - expected) < 0.02
    lq = res["logq"][:, 0].cpu()
    assert torch.allclose(lq, tl[0].log_softmax(-1)[first], atol=1e-4)


def test_adamw_matches_torch(cuda):
    torch.manual_seed(6)
    n = 10000
    p0 = torch.randn(n, device=cuda)
    g = torch.randn(n, device=cuda) * 3
    p = p0.clone()
    m = torch.zeros_like(p)
    v = torch.zeros_like(p)
    pub = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    ops.adamw_step(p, g, m, v, step=1, lr=1e-3, weight_decay=0.01, clip=1.0, publish=pub)
    ref = torch.nn.Parameter(p0.clone())
    opt = torch.optim.AdamW([ref], lr=1e-3, weight_decay=0.01)
    ref.grad = g.clone()
    torch.nn.utils.clip_grad_norm_([ref], 1.0)
    opt.step()
    assert torch.allclose(p, ref.detach(), atol=1e-6, rtol=1e-5)
    assert torch.equal(pub, p.bfloat16())


def test_status_word_clean_after_kernels(cuda):
    torch.cuda.synchronize()
    workspace.check_status(cuda)


@pytest.mark.parametrize("kind", ["tv", "forward_kl"])
def test_head_divergence_forward_backward(cuda, kind):
    torch.manual_seed(7)
    R, H, V = 12, 256, 5000
    y = torch.randn(R, H, device=cuda, requires_grad=True)
    w = (torch.randn(V, H, device=cuda) * 0.05).bfloat16()
    t = torch.randn(R, V, device=cuda) * 2
    loss = ops.head_divergence(y, w, t, kind)
    (loss * torch.arange(1, R + 1, device=cuda)).sum().backward()
    y2 = y.detach().clone().requires_grad_(True)
    log_q = (y2.bfloat16().float() @ w.float().t()).log_softmax(-1)
    log_p = t.log_softmax(-1)
    ref = 0.5 * (log_q.exp() - log_p.exp()).abs().sum(-1) if kind == "tv" else (log_p.exp() * (log_p - log_q)).sum(-1)
    (ref * torch.arange(1, R + 1, device=cuda)).sum().backward()
    assert torch.allclose(loss, ref.detach(), atol=2e-3, rtol=2e-3)
    assert _rel(y.grad, y2.grad) < 3e-2


def test_sample_arithmetic_code_point_rescaling(cuda):
    torch.manual_seed(3)
    rows, V = 6, 1000
    logits = torch.randn(rows, V, device=cuda) * 2
    inv_t = torch.full((rows,), 0.8, device=cuda)
    u = torch.rand(rows, dtype=torch.float64, device=cuda)
    arith = torch.tensor([1, 0, 1, 1, 0, 1], dtype=torch.int32, device=cuda)
    nxt = torch.full((rows,), -1.0, dtype=torch.float64, device=cuda)
    tok, _, _ = ops.sample(logits, inv_t, u, arith=arith, next_uniforms=nxt)
    rt, _, _, rn = ops.sample_reference(logits.cpu(), inv_t.cpu(), u.cpu(), with_code=True)
    torch.cuda.synchronize()
    assert torch.equal(tok.cpu(), rt)
    flagged = arith.cpu().bool()
    assert torch.allclose(nxt.cpu()[flagged], rn[flagged], atol=3e-3)   # (u - lo) / p amplifies fp32 mass error
    assert (nxt.cpu()[~flagged] == -1.0).all()
    assert ((nxt.cpu()[flagged] >= 0) & (nxt.cpu()[flagged] < 1)).all()



@pytest.mark.parametrize("B,C", [(4, 37), (64, 256), (3, 1000)])
def test_grpo_loss_kernel_matches_fp32_oracle(B, C):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + C)
    old = -torch.rand(B, C, device="cuda", generator=g) * 4
    lp = old + torch.randn(B, C, device="cuda", generator=g) * 0.3       # ratios on both sides of the clip range
    ref = old + torch.randn(B, C, device="cuda", generator=g) * 0.2
    adv = torch.randn(B, device="cuda", generator=g)
    mask = torch.rand(B, C, device="cuda", generator=g) < 0.8
    mask[0] = False                                                       # a sequence without completion tokens
    loss, grad, stats = ops.grpo_loss(lp, old, ref, adv, mask, beta=0.04, epsilon=0.2)
    want_loss, want_grad, want_stats = ops.grpo_loss_reference(lp.cpu(), old.cpu(), ref.cpu(), adv.cpu(),
                                                               mask.cpu(), beta=0.04, epsilon=0.2)
    assert torch.allclose(loss.cpu(), want_loss, rtol=1e-4, atol=1e-6)
    assert torch.allclose(grad.cpu(), want_grad, rtol=1e-4, atol=1e-8)
    assert torch.allclose(stats.cpu(), want_stats, rtol=1e-4, atol=1e-6)
    # the arrival counter resets itself: a second launch gives the same result
    loss2, _, _ = ops.grpo_loss(lp, old, ref, adv, mask, beta=0.04, epsilon=0.2)
    assert float(loss2) == float(loss)
