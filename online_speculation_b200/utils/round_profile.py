"""Run warm suffix-MH rounds, then profiler-bracketed rounds (one GPU).

    python -m online_speculation_b200.utils.round_profile [--model qwen2.5-7b] [--chains 64] \\
        [--rounds 1] [--warmup-rounds 6]

Builds the batched suffix-MH engine the way ``bench.py`` does (random-init
weights, one uniform-random prompt shared by the chains, block-4 drafts, the
online learner), extends every chain, runs ``--warmup-rounds`` rounds, then
wraps ``--rounds`` rounds in ``cudaProfilerStart`` / ``cudaProfilerStop`` so a
profiler started with ``--profile-from-start off`` sees exactly those rounds'
kernel launches (for example ``ncu --metrics gpu__time_duration.sum
--clock-control none --profile-from-start off --csv ...``).  Prints one JSON
line with the device time of the bracketed rounds (CUDA events; not meaningful
under a profiler).
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
    a = p.parse_args(argv)

    import numpy as np
    import torch

    from ..api import build_mh_engine

    torch.cuda.set_device(0)
    eng = build_mh_engine(a.model, tp_group=None, seed=a.seed, alpha=4.0, length=a.gen_len, block_size=a.block,
                          learner_stride=a.stride, use_graphs=True, kv_bytes=24 << 30,
                          max_seq_tokens=a.prompt_len + a.gen_len + 2 * a.block)
    rng = np.random.default_rng(a.seed + 17)
    prompt = rng.integers(0, eng.runner.cfg.vocab_size - 2, size=a.prompt_len).tolist()
    eng.add_chains([prompt] * a.chains)
    eng.run_until_idle()
    eng.set_quota(a.warmup_rounds + a.rounds + 64)
    for _ in range(a.warmup_rounds):
        eng.round()
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()
    t0.record()
    for _ in range(a.rounds):
        eng.round()
    t1.record()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"rounds": a.rounds, "ms_per_round": t0.elapsed_time(t1) / a.rounds,
                      "learner_updates": eng.learner.updates if eng.learner else 0}))
    eng.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
