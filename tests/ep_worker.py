"""Worker for tests/test_ep_gpu.py (launched with torch.distributed.run).

Every rank holds the full random expert weights, routes its own tokens and
checks the fused expert-parallel layer and the NCCL all-to-all baseline
against the single-GPU MoE layer on the same tokens.
"""

import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from online_speculation_b200.ops import kernels as K  # noqa: E402
from online_speculation_b200.ops import workspace  # noqa: E402
from online_speculation_b200.parallel.ep import ExpertParallelMoE, NcclExpertParallelMoE  # noqa: E402


def rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm())


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = torch.device("cuda", local)
    E, k, H, F = 16, 4, 256, 128
    El = E // world
    g = torch.Generator(device=dev).manual_seed(5)
    router = (torch.randn(E, H, device=dev, generator=g) * 0.05).bfloat16()
    w_gu = (torch.randn(E * 2 * F, H, device=dev, generator=g) * 0.05).bfloat16()
    w_down = (torch.randn(E * H, F, device=dev, generator=g) * 0.05).bfloat16()
    gu_local = w_gu[rank * El * 2 * F:(rank + 1) * El * 2 * F].contiguous()
    down_local = w_down[rank * El * H:(rank + 1) * El * H].contiguous()
    fused = ExpertParallelMoE(dist.group.WORLD, experts=E, top_k=k, hidden=H, ffn=F, max_tokens=512, device=dev)
    nccl = NcclExpertParallelMoE(dist.group.WORLD, experts=E, top_k=k, hidden=H, ffn=F, max_tokens=512, device=dev)
    for it in range(3):
        T = 200 + 37 * rank + 11 * it
        gt = torch.Generator(device=dev).manual_seed(100 * rank + it)
        x = torch.randn(T, H, device=dev, generator=gt).bfloat16()
        h = torch.randn(T, H, device=dev, generator=gt).bfloat16()
        ref = K.moe_ffn(x, h.clone(), router, w_gu, w_down, top_k=k)
        a = fused.ffn(x, h.clone(), router, gu_local, down_local)
        b = nccl.ffn(x, h.clone(), router, gu_local, down_local)
        torch.cuda.synchronize()
        delta = (ref.float() - h.float())
        assert rel(a.float() - h.float(), delta) < 1e-2, ("fused", it, rel(a.float() - h.float(), delta))
        assert rel(b.float() - h.float(), delta) < 1e-2, ("nccl", it, rel(b.float() - h.float(), delta))
    workspace.check_status(dev)
    dist.barrier()
    if rank == 0:
        print("EP_OK", world, flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
