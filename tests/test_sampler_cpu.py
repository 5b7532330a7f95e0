"""Truncated sampling policies (CPU oracle): top-k / top-p kept sets, normalisation and draws."""

import numpy as np
import torch

from online_speculation_b200.ops import kernels as ops


def _kept_numpy(z, k, p):
    """Kept columns of one row by explicit sorting (the policy's definition)."""
    order = np.argsort(-z, kind="stable")
    keep = np.ones_like(z, dtype=bool)
    if 0 < k < z.size:
        keep &= z >= z[order[k - 1]]
    if p < 1:
        zz = np.where(keep, z, -np.inf)
        order = np.argsort(-zz, kind="stable")
        probs = np.exp(zz[order] - zz[order[0]])
        probs /= probs.sum()
        before = np.concatenate(([0.0], np.cumsum(probs)[:-1]))
        drop = np.zeros_like(keep)
        drop[order] = before > p
        keep &= ~drop
    return keep


def test_truncated_log_policy_matches_sorting_definition():
    g = torch.Generator().manual_seed(0)
    z = torch.randn(24, 300, generator=g, dtype=torch.float32) * 2
    ks = torch.tensor([0, 1, 3, 10, 299, 300] * 4, dtype=torch.int32)
    ps = torch.tensor([1.0, 0.5, 0.9, 0.2] * 6, dtype=torch.float32)
    log_q = ops.truncated_log_policy(z.clone(), ks, ps)
    for r in range(24):
        keep = _kept_numpy(z[r].double().numpy(), int(ks[r]), float(ps[r]))
        got = torch.isfinite(log_q[r]).numpy()
        assert np.array_equal(got, keep)
        assert abs(float(log_q[r][got].exp().sum()) - 1.0) < 1e-5
        zk = z[r][torch.from_numpy(keep)]
        assert torch.allclose(log_q[r][got], zk - torch.logsumexp(zk, 0), atol=1e-5)


def test_sample_reference_draws_inside_the_kept_set():
    g = torch.Generator().manual_seed(1)
    logits = torch.randn(64, 500, generator=g) * 3
    ks = torch.tensor([0, 5, 40, 0] * 16, dtype=torch.int32)
    ps = torch.tensor([0.3, 1.0, 0.8, 0.95] * 16, dtype=torch.float32)
    u = torch.rand(64, generator=g, dtype=torch.float64)
    tok, lq, lp = ops.sample_reference(logits, None, u, top_k=ks, top_p=ps)
    log_q = ops.truncated_log_policy(logits, ks, ps)
    assert bool(torch.isfinite(log_q.gather(-1, tok.long()[:, None])).all())
    assert torch.allclose(lq, log_q.gather(-1, tok.long()[:, None]).squeeze(-1))
    assert torch.allclose(lp, logits.log_softmax(-1).gather(-1, tok.long()[:, None]).squeeze(-1))
    # the same uniforms through the CPU dispatch of ops.sample give the same draws
    t2, q2, _ = ops.sample(logits, None, u, top_k=ks, top_p=ps)
    assert torch.equal(t2, tok) and torch.allclose(q2, lq)


def test_row_stats_truncated_cpu_scores_outside_as_minus_inf():
    logits = torch.tensor([[3.0, 2.0, 1.0, 0.0]])
    _, lse_t, _, logq = ops.row_stats(logits, None, torch.tensor([3], dtype=torch.int32),
                                      top_k=torch.tensor([2], dtype=torch.int32))
    assert logq.item() == float("-inf")
    assert abs(lse_t.item() - float(torch.logsumexp(torch.tensor([3.0, 2.0]), 0))) < 1e-6
