"""GRPO on the sm_100a kernels: training ops against fp32 PyTorch, trainer gradients, a full step."""

import pytest
import torch

from online_speculation_b200.ops import kernels as ops

pytestmark = pytest.mark.gpu


def test_kernel_linear_forward_backward():
    torch.manual_seed(0)
    x = torch.randn(300, 256, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(384, 256, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_(True)
    b = (torch.randn(384, device="cuda") * 0.1).to(torch.bfloat16).requires_grad_(True)
    y = ops.kernel_linear(x, w, b)
    gy = torch.randn_like(y)
    y.backward(gy)
    xf, wf, bf = (t.detach().float().requires_grad_(True) for t in (x, w, b))
    yf = xf @ wf.t() + bf
    yf.backward(gy.float())
    assert (y.float() - yf).abs().max() < 0.05
    for got, ref in ((x.grad, xf.grad), (w.grad, wf.grad), (b.grad, bf.grad)):
        assert (got.float() - ref).norm() / ref.norm() < 0.01


@pytest.mark.parametrize("chunk", [64, 1000])
def test_head_logprob_matches_fp32(chunk):
    torch.manual_seed(1)
    R, H, V = 200, 256, 5000
    h = torch.randn(R, H, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(V, H, device="cuda") * 0.1).to(torch.bfloat16).requires_grad_(True)
    t = torch.randint(0, V, (R,), device="cuda")
    lp = ops.head_logprob(h, w, t, chunk_rows=chunk)
    g = torch.randn(R, device="cuda")
    lp.backward(g)
    hf, wf = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    ref = (hf @ wf.t()).log_softmax(-1).gather(-1, t[:, None]).squeeze(-1)
    ref.backward(g)
    assert (lp - ref).abs().max() < 2e-2
    assert (h.grad.float() - hf.grad).norm() / hf.grad.norm() < 0.02
    assert (w.grad.float() - wf.grad).norm() / wf.grad.norm() < 0.02


def test_target_logprob_matches_fp32():
    torch.manual_seed(2)
    logits = torch.randn(64, 3001, device="cuda", requires_grad=True)
    t = torch.randint(0, 3001, (64,), device="cuda")
    lp = ops.target_logprob(logits, t)
    g = torch.randn(64, device="cuda")
    lp.backward(g)
    lf = logits.detach().clone().requires_grad_(True)
    ref = lf.log_softmax(-1).gather(-1, t[:, None]).squeeze(-1)
    ref.backward(g)
    assert (lp - ref).abs().max() < 1e-4
    assert (logits.grad - lf.grad).abs().max() < 1e-5


def test_grpo_gradients_match_fp32_oracle_on_gpu():
    from online_speculation_b200.models.decoder import build_weights, random_state_dict
    from online_speculation_b200.training.grpo import GRPOConfig, GRPOTrainer, group_advantages
    from test_grpo_cpu import TINY, _oracle_grads

    sd = random_state_dict(TINY, seed=3, std=0.05)
    conf = GRPOConfig(group_size=2, prompt_length=16, completion_length=48, head_chunk_rows=40)
    tr = GRPOTrainer(TINY, conf, device="cuda", rollouts=False, state_dict={k: v.cuda() for k, v in sd.items()})
    ids = torch.randint(0, TINY.vocab_size, (2, 64), generator=torch.Generator().manual_seed(1))
    mask = torch.ones(2, 48, dtype=torch.bool)
    mask[0, 40:] = False
    rewards = torch.tensor([0.0, 1.0])
    grad, _ = tr.compute_gradients(ids.cuda(), mask.cuda(), rewards.cuda())
    oracle = _oracle_grads(TINY, sd, ids, 16, group_advantages(rewards, 2), mask)
    mapped = build_weights(TINY, oracle, dtype=torch.float32)
    checks = {"embed": mapped.embed, "final_norm": mapped.final_norm}
    for i, lw in enumerate(mapped.layers):
        for f in ("in_norm", "post_norm", "w_qkv", "b_qkv", "w_o", "w_gu", "w_down"):
            checks[f"{i}.{f}"] = getattr(lw, f)
    for name, ref in checks.items():
        got = tr.params.view(name, grad).cpu()
        err = (got - ref).norm() / ref.norm().clamp(min=1e-12)
        assert err < 0.05, (name, float(err))


def test_grpo_step_with_rollouts():
    from online_speculation_b200.models.decoder import DecoderConfig
    from online_speculation_b200.training.grpo import GRPOConfig, GRPOTrainer

    cfg = DecoderConfig(vocab_size=2048, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                        num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=True, name="small")
    conf = GRPOConfig(group_size=4, prompts_per_rank=2, prompt_length=32, completion_length=64,
                      learning_rate=1e-4)
    tr = GRPOTrainer(cfg, conf, kv_bytes=1 << 28)
    try:
        before = tr.parameter("1.w_down").clone()
        s1 = tr.step()
        s2 = tr.step()
        assert s1["tokens"] == 8 * 96 and s2["step"] == 2
        assert tr.check_finite()
        assert not torch.equal(before, tr.parameter("1.w_down"))
        assert s2["kl"] >= 0 and s2["kl"] < 1.0
    finally:
        tr.close()
