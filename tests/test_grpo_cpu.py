"""GRPO trainer on CPU: loss maths, gradients against an fp32 autograd oracle, data-parallel sharding (gloo)."""

import os

import pytest
import torch

from online_speculation_b200.models.decoder import DecoderConfig, build_weights, random_state_dict, reference_forward
from online_speculation_b200.training.grpo import GRPOConfig, GRPOTrainer, group_advantages, grpo_loss

TINY = DecoderConfig(vocab_size=256, hidden_size=128, intermediate_size=128, num_hidden_layers=2,
                     num_attention_heads=2, num_key_value_heads=1, tie_word_embeddings=True, name="t")


def test_group_advantages():
    r = torch.tensor([1.0, 0.0, 1.0, 1.0, 0.0, 0.0, 0.0, 1.0])
    a = group_advantages(r, 4)
    assert torch.allclose(a, torch.tensor([0.25, -0.75, 0.25, 0.25, -0.25, -0.25, -0.25, 0.75]))
    s = group_advantages(r, 4, "group")
    assert torch.allclose(s.view(2, 4).std(1), torch.ones(2), atol=1e-3)


def test_grpo_loss_ratio_one_gradient():
    torch.manual_seed(0)
    lp = torch.randn(2, 5, requires_grad=True)
    ref = lp.detach() + 0.1 * torch.randn(2, 5)
    adv = torch.tensor([0.5, -0.5])
    mask = torch.ones(2, 5, dtype=torch.bool)
    mask[1, 3:] = False
    loss, info = grpo_loss(lp, lp.detach(), ref, adv, mask, beta=0.04, epsilon=0.2)
    loss.backward()
    # d/dlp of -(A - beta (e^{ref-lp} - (ref-lp) - 1)) / n / B
    n = mask.float().sum(1, keepdim=True)
    d = ref - lp.detach()
    expect = -(adv[:, None] - 0.04 * (-torch.exp(d) + 1)) / n / 2 * mask
    assert torch.allclose(lp.grad, expect, atol=1e-6)
    assert info["clip_fraction"] == 0.0


def _oracle_grads(cfg, sd, ids, prompt_len, adv, mask):
    """fp32 autograd of the ratio-one GRPO loss (KL gradient is zero at ref = policy)."""
    f = {k: v.float().requires_grad_(True) for k, v in sd.items()}
    B = ids.shape[0]
    terms = []
    for b in range(B):
        logits = reference_forward(cfg, f, ids[b])
        lp = logits[prompt_len - 1:-1].log_softmax(-1).gather(-1, ids[b, prompt_len:, None]).squeeze(-1)
        m = mask[b].float()
        terms.append((adv[b] * lp * m).sum() / m.sum())
    loss = -torch.stack(terms).mean()
    loss.backward()
    return {k: v.grad if v.grad is not None else torch.zeros_like(v) for k, v in f.items()}


def test_gradients_match_fp32_oracle():
    cfg = TINY
    sd = random_state_dict(cfg, seed=3, std=0.05)
    conf = GRPOConfig(group_size=2, prompts_per_rank=1, prompt_length=6, completion_length=10, head_chunk_rows=7)
    tr = GRPOTrainer(cfg, conf, device="cpu", rollouts=False, state_dict=sd)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (2, 16), generator=g)
    mask = torch.ones(2, 10, dtype=torch.bool)
    mask[1, 7:] = False
    rewards = torch.tensor([1.0, 0.0])
    grad, info = tr.compute_gradients(ids, mask, rewards)
    oracle = _oracle_grads(cfg, sd, ids, 6, group_advantages(rewards, 2), mask)
    mapped = build_weights(cfg, oracle, dtype=torch.float32)
    checks = {"embed": mapped.embed, "final_norm": mapped.final_norm}
    for i, lw in enumerate(mapped.layers):
        for f in ("in_norm", "post_norm", "w_qkv", "b_qkv", "w_o", "w_gu", "w_down"):
            checks[f"{i}.{f}"] = getattr(lw, f)
    for name, ref in checks.items():
        got = tr.params.view(name, grad)
        err = (got - ref).norm() / ref.norm().clamp(min=1e-12)
        assert err < 0.05, (name, float(err))
    assert info["kl"] == pytest.approx(0.0, abs=1e-6)


def test_optimizer_step_moves_parameters():
    conf = GRPOConfig(group_size=2, prompts_per_rank=1, prompt_length=4, completion_length=4, learning_rate=1e-3)
    tr = GRPOTrainer(TINY, conf, device="cpu", rollouts=False, seed=2)
    before = tr.parameter("0.w_o").clone()
    ids = torch.randint(0, TINY.vocab_size, (2, 8), generator=torch.Generator().manual_seed(0))
    tr.train_on(ids, torch.ones(2, 4, dtype=torch.bool), torch.tensor([1.0, 0.0]))
    after = tr.parameter("0.w_o")
    assert not torch.equal(before, after)
    assert tr.step_count == 1 and torch.isfinite(tr.master).all()


def _dp_worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        conf = GRPOConfig(group_size=2, prompts_per_rank=1, prompt_length=4, completion_length=6)
        tr = GRPOTrainer(TINY, conf, device="cpu", rollouts=False, seed=5, group=dist.group.WORLD)
        ids = torch.randint(0, TINY.vocab_size, (2 * world, 10), generator=torch.Generator().manual_seed(7))
        rewards = torch.tensor([1.0, 0.0, 0.0, 1.0, 1.0, 1.0, 0.0, 0.0][: 2 * world])
        mask = torch.ones(2 * world, 6, dtype=torch.bool)
        g, _ = tr.compute_gradients(ids[2 * rank:2 * rank + 2], mask[:2], rewards[2 * rank:2 * rank + 2])
        shard = g.clone()
        tr._optimizer_step(g)
        # numpy copies travel by value: a tensor would be passed through shared memory owned by
        # this process, which may have exited before the parent unpickles it
        q.put((rank, shard.float().numpy().copy(), tr.params.shard_ranges(), tr.params.flat.float().numpy()))
    finally:
        dist.destroy_process_group()


def test_data_parallel_sharded_gradients_and_allgather():
    import torch.multiprocessing as mp

    from online_speculation_b200.training.grpo import FlatParameters, _named_tensors

    from conftest import free_port

    world, port = 2, free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=240) for _ in range(world)], key=lambda x: x[0])
    res = [(r, torch.from_numpy(shard), ranges, torch.from_numpy(flat)) for r, shard, ranges, flat in res]
    for p in procs:
        p.join(timeout=60)
    assert torch.equal(res[0][3], res[1][3]), "all-gathered parameters differ across ranks"
    # the data-parallel gradient, reassembled from the shards in the world-2 layout
    layout = FlatParameters(_named_tensors(build_weights(TINY, random_state_dict(TINY, seed=5))), world, 0, "cpu")
    dp = torch.zeros(layout.numel, dtype=torch.float32)
    for _, shard, ranges, _ in res:
        for lo, hi, pos in ranges:
            dp[lo:hi] = shard[pos:pos + hi - lo]
    # single-process oracle on the union of the ranks' batches (groups are not split across ranks)
    conf = GRPOConfig(group_size=2, prompts_per_rank=world, prompt_length=4, completion_length=6)
    one = GRPOTrainer(TINY, conf, device="cpu", rollouts=False, seed=5)
    ids = torch.randint(0, TINY.vocab_size, (2 * world, 10), generator=torch.Generator().manual_seed(7))
    full, _ = one.compute_gradients(ids, torch.ones(2 * world, 6, dtype=torch.bool),
                                    torch.tensor([1.0, 0.0, 0.0, 1.0]))
    for name in one.params.slots:
        a, b = layout.view(name, dp), one.params.view(name, full)
        err = (a - b).norm() / b.norm().clamp(min=1e-12)
        assert err < 1e-2, (name, float(err))   # bf16 reductions over different row counts


def _synthetic(step):
    g = torch.Generator().manual_seed(100 + step)
    ids = torch.randint(0, TINY.vocab_size, (4, 10), generator=g)
    rewards = (torch.rand(4, generator=g) < 0.5).float()
    return ids, torch.ones(4, 6, dtype=torch.bool), rewards


def test_grpo_run_checkpoints_resume_bit_exact_and_refuse_changed_settings(tmp_path):
    import json

    from online_speculation_b200.training.grpo_run import GRPORun, latest_checkpoint

    conf = GRPOConfig(group_size=2, prompts_per_rank=2, prompt_length=4, completion_length=6, learning_rate=1e-3)
    straight = GRPORun(tmp_path / "a", TINY, conf, max_steps=4, save_steps=2, device="cpu", seed=3, data=_synthetic)
    straight.train()
    assert latest_checkpoint(tmp_path / "a").name == "checkpoint-4"
    assert (tmp_path / "a" / "checkpoint-2" / "rank0.pt").is_file()
    manifest = json.loads((tmp_path / "a" / "run_manifest.json").read_text())
    assert manifest["status"] == "completed" and manifest["final_step"] == 4
    # an interrupted run (2 steps) continued to 4 steps reaches the same parameters
    first = GRPORun(tmp_path / "b", TINY, conf, max_steps=2, save_steps=2, device="cpu", seed=3, data=_synthetic)
    first.train()
    second = GRPORun(tmp_path / "b", TINY, conf, max_steps=4, save_steps=2, device="cpu", seed=3, data=_synthetic)
    assert second.resumed_from.endswith("checkpoint-2") and second.trainer.step_count == 2
    second.train()
    assert torch.equal(second.trainer.params.flat, straight.trainer.params.flat)
    assert torch.equal(second.trainer.master, straight.trainer.master)
    # other hyper-parameters in the same directory are refused; more steps are not
    other = GRPOConfig(group_size=2, prompts_per_rank=2, prompt_length=4, completion_length=6, learning_rate=2e-3)
    with pytest.raises(ValueError, match="different"):
        GRPORun(tmp_path / "b", TINY, other, max_steps=4, device="cpu", seed=3, data=_synthetic)
    fresh = GRPORun(tmp_path / "b", TINY, conf, max_steps=6, save_steps=2, device="cpu", seed=3, data=_synthetic,
                    resume="none")
    assert fresh.trainer.step_count == 0


def test_grpo_loss_cpu_matches_the_kernel_oracle():
    from online_speculation_b200.ops import kernels as K
    from online_speculation_b200.training.grpo import grpo_loss

    g = torch.Generator().manual_seed(3)
    old = -torch.rand(5, 19, generator=g) * 3
    lp = (old + torch.randn(5, 19, generator=g) * 0.3).requires_grad_(True)
    ref = old + torch.randn(5, 19, generator=g) * 0.2
    adv = torch.randn(5, generator=g)
    mask = torch.rand(5, 19, generator=g) < 0.7
    loss, info = grpo_loss(lp, old, ref, adv, mask, beta=0.04, epsilon=0.2)
    loss.backward()
    want, grad, stats = K.grpo_loss_reference(lp, old, ref, adv, mask, beta=0.04, epsilon=0.2)
    assert torch.allclose(loss.detach(), want) and torch.allclose(lp.grad, grad)
    assert info["kl"] == pytest.approx(float(stats[1]), rel=1e-6)
    assert info["clip_fraction"] == pytest.approx(float(stats[2]), rel=1e-6)
