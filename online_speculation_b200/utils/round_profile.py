"""Run warm suffix-MH rounds, then profiler-bracketed rounds (one GPU).

    python -m online_speculation_b200.utils.round_profile [--model qwen2.5-7b] [--chains 64] \\
        [--rounds 1] [--warmup-rounds 6] [--policy always|never|adaptive] [--plain-steps 4]

Builds the batched suffix-MH engine the way ``bench.py`` does (random-init
weights, one uniform-random prompt shared by the chains, block-4 drafts, the
online learner), extends every chain, runs ``--warmup-rounds`` rounds, then
wraps ``--rounds`` rounds in ``cudaProfilerStart`` / ``cudaProfilerStop`` so a
profiler started with ``--profile-from-start off`` sees exactly those rounds'
kernel launches (for example ``ncu --metrics gpu__time_duration.sum
--clock-control none --profile-from-start off --csv ...``).  Prints one JSON
line with the device time of the bracketed rounds (CUDA events; not meaningful
under a profiler).  Under ``torch.distributed.run`` (WORLD_SIZE > 1) the engine is
tensor parallel over the ranks.  ``--kernel-table`` records the bracketed rounds'
kernels through the CUDA activity trace instead (no kernel replay, so it may run
on every rank) and writes one device-time table per rank.
"""

from __future__ import annotations

import argparse
import json


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.utils.round_profile")
    p.add_argument("--model", default="qwen2.5-7b")
    p.add_argument("--chains", type=int, default=64)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--gen-len", type=int, default=512)
    p.add_argument("--block", type=int, default=4)
    p.add_argument("--stride", type=int, default=64, help="learner stride in verified blocks")
    p.add_argument("--rounds", type=int, default=1)
    p.add_argument("--warmup-rounds", type=int, default=6)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--policy", choices=("always", "never", "adaptive"), default="always",
                   help="speculation policy of the engine (never: plain decode rounds only)")
    p.add_argument("--plain-steps", type=int, default=4)
    p.add_argument("--no-pdl", action="store_true",
                   help="launch without programmatic dependent launch, so each kernel's traced duration is its "
                        "own (with it, a kernel's span includes its wait for the predecessor)")
    p.add_argument("--kernel-table", help="write a per-kernel device-time table of the bracketed rounds "
                                          "(CUDA activity trace through torch.profiler) to this JSON file; "
                                          "{rank} in the name is replaced by the rank")
    a = p.parse_args(argv)

    import numpy as np
    import torch

    from ..api import build_mh_engine

    import os

    group, rank, world = None, 0, int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        group, rank = dist.group.WORLD, dist.get_rank()
    else:
        torch.cuda.set_device(0)
    if a.no_pdl:
        from ..ops import _ext

        _ext.require().set_pdl(False)
    eng = build_mh_engine(a.model, tp_group=group, seed=a.seed, alpha=4.0, length=a.gen_len, block_size=a.block,
                          learner_stride=a.stride, use_graphs=True, kv_bytes=24 << 30,
                          max_seq_tokens=a.prompt_len + a.gen_len + 2 * a.block, spec_policy=a.policy,
                          plain_steps=a.plain_steps)
    rng = np.random.default_rng(a.seed + 17)
    prompt = rng.integers(0, eng.runner.cfg.vocab_size - 2, size=a.prompt_len).tolist()
    eng.add_chains([prompt] * a.chains)
    eng.run_until_idle()
    eng.set_quota(a.warmup_rounds + a.rounds + 64)
    for _ in range(a.warmup_rounds):
        eng.round()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    trace = None
    if a.kernel_table:
        from torch.profiler import ProfilerActivity, profile

        trace = profile(activities=[ProfilerActivity.CUDA])
        trace.__enter__()
    else:
        torch.cuda.profiler.start()
    t0.record()
    for _ in range(a.rounds):
        eng.round()
    t1.record()
    torch.cuda.synchronize()
    if trace is not None:
        trace.__exit__(None, None, None)
        table: dict = {}
        for ev in trace.events():
            if ev.device_type.name != "CUDA":
                continue
            row = table.setdefault(ev.name, [0, 0.0])
            row[0] += 1
            row[1] += ev.time_range.elapsed_us()
        rows = sorted(({"kernel": k, "count": c, "us": round(t, 1)} for k, (c, t) in table.items()),
                      key=lambda r: -r["us"])
        with open(a.kernel_table.replace("{rank}", str(rank)), "w", encoding="utf-8") as handle:
            json.dump({"rank": rank, "world": world, "rounds": a.rounds, "kernels": rows}, handle, indent=1)
    else:
        torch.cuda.profiler.stop()
    if rank == 0:
        print(json.dumps({"rounds": a.rounds, "policy": a.policy, "world": world,
                          "ms_per_round": t0.elapsed_time(t1) / a.rounds,
                          "learner_updates": eng.learner.updates if eng.learner else 0}))
    eng.close()
    if group is not None:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
