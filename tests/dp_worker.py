"""Worker for tests/test_dp_gpu.py (launched with torch.distributed.run).

Checks the peer-memory data-parallel kernels against NCCL on every rank:
reduce-scatter of rank-specific gradients over several buckets (bit-exact against the
rank-order fp32 sum), all-gather of rank-specific bf16 shards (exact), both repeated so
the call counters advance; then one GRPO optimisation step with the peer-memory
collectives against the same step with NCCL.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from online_speculation_b200.models.decoder import DecoderConfig  # noqa: E402
from online_speculation_b200.ops import workspace  # noqa: E402
from online_speculation_b200.parallel.dp import SymmetricDataParallel  # noqa: E402
from online_speculation_b200.training.grpo import GRPOConfig, GRPOTrainer  # noqa: E402

TINY = DecoderConfig(vocab_size=256, hidden_size=128, intermediate_size=128, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, name="tiny")


def kernels(rank, world, dev):
    dp = SymmetricDataParallel(dist.group.WORLD, dev, wait_limit_ns=2_000_000_000)
    quantum = world * 64
    buckets = [(0, 3 * quantum), (3 * quantum, 10 * quantum), (10 * quantum, 11 * quantum)]
    numel = buckets[-1][1]
    grad = dp.allocate(numel, torch.float32)
    params = dp.allocate(numel, torch.bfloat16)
    side = torch.cuda.Stream(device=dev)
    for it in range(3):
        g = torch.Generator(device=dev).manual_seed(1000 * it + rank)
        grad.copy_(torch.randn(numel, device=dev, generator=g))
        every = [torch.empty_like(grad) for _ in range(world)]
        dist.all_gather(every, grad)
        for lo, hi in buckets:
            n = (hi - lo) // world
            shard = torch.empty(n, dtype=torch.float32, device=dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(side):
                dp.reduce_scatter(grad, lo, hi, shard, 1.0 / world)
            torch.cuda.current_stream(dev).wait_stream(side)
            acc = every[0][lo + rank * n:lo + (rank + 1) * n].clone()
            for q in range(1, world):
                acc += every[q][lo + rank * n:lo + (rank + 1) * n]
            assert torch.equal(shard, acc * (1.0 / world)), f"reduce-scatter differs (iteration {it})"
        src_all = torch.arange(numel, device=dev, dtype=torch.float32).remainder(251).add(it).to(torch.bfloat16)
        for lo, hi in buckets:
            n = (hi - lo) // world
            mine = src_all[lo + rank * n:lo + (rank + 1) * n].contiguous()
            dp.all_gather(params, lo, hi, mine)
        torch.cuda.synchronize(dev)
        assert torch.equal(params, src_all), f"all-gather differs (iteration {it})"
        dist.barrier()
    workspace.check_status(dev)


def grpo(rank, world, dev):
    ids = torch.randint(0, TINY.vocab_size, (2 * world, 10), generator=torch.Generator().manual_seed(7)).to(dev)
    rewards = torch.tensor([1.0, 0.0, 0.0, 1.0, 1.0, 1.0, 0.0, 0.0] * 2, device=dev)[: 2 * world]
    mask = torch.ones(2, 6, dtype=torch.bool, device=dev)
    out = {}
    for kind in ("nccl", "symmetric"):
        conf = GRPOConfig(group_size=2, prompts_per_rank=1, prompt_length=4, completion_length=6, learning_rate=1e-3,
                          dp_collectives=kind)
        tr = GRPOTrainer(TINY, conf, device=dev, rollouts=False, seed=5, group=dist.group.WORLD)
        assert (tr.dp.symmetric) == (kind == "symmetric")
        losses = []
        for _ in range(2):
            info = tr.train_on(ids[2 * rank:2 * rank + 2], mask, rewards[2 * rank:2 * rank + 2])
            losses.append(info["loss"])
        torch.cuda.synchronize(dev)
        workspace.check_status(dev)
        out[kind] = (losses, tr.master.clone(), tr.params.flat.clone())
    (l0, m0, f0), (l1, m1, f1) = out["nccl"], out["symmetric"]
    assert abs(l0[0] - l1[0]) < 1e-6, (l0, l1)
    # NCCL may sum the ranks in another order: the fp32 gradients agree to rounding, AdamW's first
    # steps follow their signs, so the masters agree except where a gradient is ~0
    close = (m0 - m1).abs() <= 1e-6 + 1e-3 * m0.abs()
    assert float(close.float().mean()) > 0.999, float(close.float().mean())
    # every rank holds the same all-gathered parameters
    every = [torch.empty_like(f1) for _ in range(world)]
    dist.all_gather(every, f1)
    assert all(torch.equal(every[0], e) for e in every)


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    try:
        kernels(rank, world, dev)
        grpo(rank, world, dev)
        dist.barrier()
        if rank == 0:
            print("DP_OK", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
