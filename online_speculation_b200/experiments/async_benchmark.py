"""Synchronous against continuously batched execution of the inference-scaling methods.

For every method, the same prompts and seeds run twice on one backend:

* ``synchronous`` -- one prompt after another, each method call issuing its own
  ``sample_batch`` / ``score_batch`` calls;
* ``asynchronous`` -- ``--workers`` threads run the prompts concurrently behind a
  :class:`~online_speculation_b200.arllm.backends.batching.ContinuousBatchingBackend`,
  which merges the threads' calls into wide backend calls.

Both arms sit behind a score cache of their own, as in the reference.  Each arm reports wall
and device seconds and the backend's counters; the asynchronous arm adds the batching
wrapper's statistics (merged calls, widest batch) and the agreement of its outputs with the
synchronous ones: every request carries its own seed and uniforms, so batching changes
which call computes a token but not which token is drawn, up to logits that differ between
batch widths in their last bits (which can move a draw on a near-flat law).

    python -m online_speculation_b200.experiments.async_benchmark --output async.json \\
        [--model random:qwen2.5-0.5b] [--methods conditional_is,reward_mh,best_of_n] \\
        [--prompts 8] [--workers 8] [--max-new-tokens 32]

Purpose and arm layout of experiments/arllm/gsm8k_async_benchmark.py; the GSM8K problems
and verifier are replaced by uniform-random prompts and a sequence-log-probability reward.
"""

from __future__ import annotations

import argparse
import json
from collections.abc import Callable, Sequence
from concurrent.futures import ThreadPoolExecutor
from dataclasses import asdict, is_dataclass
from pathlib import Path
from typing import Any

import numpy as np

from ..arllm.backends.batching import ContinuousBatchingBackend
from ..arllm.backends.cache import ScoreCachingBackend
from .methods import MethodSettings, run_ar_method
from .rollout_infra import agreement, counter_delta, measure

DEFAULT_METHODS = ("best_of_n", "reward_mh", "conditional_is")


def _plain(snapshot: Any) -> dict:
    if snapshot is None:
        return {}
    return asdict(snapshot) if is_dataclass(snapshot) and not isinstance(snapshot, type) else dict(snapshot)


def run_benchmark(backend, *, prompts: Sequence[tuple], methods: Sequence[str] = DEFAULT_METHODS,
                  settings: MethodSettings | None = None, workers: int = 8, seed: int = 20260812,
                  reward_factory: Callable[[Any], Callable] | None = None, max_batch_size: int = 64,
                  max_batch_tokens: int = 1 << 16) -> dict:
    settings = settings or MethodSettings()
    snap = getattr(backend, "snapshot", lambda: None)
    report: dict[str, Any] = {"workload": {"prompts": len(prompts), "prompt_tokens": [len(p) for p in prompts],
                                           "workers": workers, "methods": list(methods), "seed": seed,
                                           "settings": asdict(settings)}, "methods": {}}
    for method in methods:
        seeds = [int(np.random.SeedSequence([seed, i]).generate_state(1)[0]) for i in range(len(prompts))]

        def run_sync():
            cached = ScoreCachingBackend(backend)
            reward = reward_factory(cached) if reward_factory else None
            return [run_ar_method(method, cached, p, settings, s, reward=reward) for p, s in zip(prompts, seeds)]

        def run_async():
            wrapper = ContinuousBatchingBackend(backend, max_batch_size=max_batch_size,
                                                max_batch_tokens=max_batch_tokens)
            try:
                cached = ScoreCachingBackend(wrapper)
                reward = reward_factory(cached) if reward_factory else None
                with ThreadPoolExecutor(max_workers=max(1, min(workers, len(prompts)))) as pool:
                    outs = list(pool.map(lambda ps: run_ar_method(method, cached, ps[0], settings, ps[1],
                                                                  reward=reward), zip(prompts, seeds)))
                return outs, _plain(wrapper.snapshot())
            finally:
                wrapper.close()

        before = snap()
        sync_out, ts = measure(run_sync)
        mid = snap()
        (async_out, batching), ta = measure(run_async)
        after = snap()
        tokens_s = sum(len(o.token_ids) for o in sync_out)
        tokens_a = sum(len(o.token_ids) for o in async_out)
        sync_ids = {str(i): tuple(o.token_ids) for i, o in enumerate(sync_out)}
        async_ids = {str(i): tuple(o.token_ids) for i, o in enumerate(async_out)}
        report["methods"][method] = {
            "synchronous": {"telemetry": ts, "main_model": counter_delta(before, mid), "output_tokens": tokens_s},
            "asynchronous": {"telemetry": ta, "main_model": counter_delta(mid, after), "output_tokens": tokens_a,
                             "batching": batching, "agreement_with_synchronous": agreement(async_ids, sync_ids)},
            "speedup": ts["device_seconds"] / ta["device_seconds"] if ta["device_seconds"] else None,
        }
    return report


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.async_benchmark")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--model", default="random:qwen2.5-0.5b", help="random:<preset> or a local checkpoint directory")
    p.add_argument("--methods", default=",".join(DEFAULT_METHODS))
    p.add_argument("--prompts", type=int, default=8)
    p.add_argument("--prompt-tokens", type=int, default=64)
    p.add_argument("--workers", type=int, default=8)
    p.add_argument("--max-new-tokens", type=int, default=32)
    p.add_argument("--block-size", type=int, default=8)
    p.add_argument("--kv-cache-gb", type=float, default=8.0)
    p.add_argument("--seed", type=int, default=20260812)
    a = p.parse_args(argv)

    from ..arllm.backends.loader import LoadedModel
    from ..arllm.rewards import SequenceLogProbabilityReward

    backend = LoadedModel(a.model, {"runtime": {"kv_cache_gb": a.kv_cache_gb, "max_batch_size": 64,
                                                "max_sequence_tokens": a.prompt_tokens + 2 * a.max_new_tokens + 64}},
                          "base").backend
    try:
        rng = np.random.default_rng(a.seed)
        prompts = [tuple(int(t) for t in rng.integers(0, backend.vocab_size, a.prompt_tokens))
                   for _ in range(a.prompts)]
        settings = MethodSettings(max_new_tokens=a.max_new_tokens, block_size=a.block_size)
        report = run_benchmark(backend, prompts=prompts, methods=[m for m in a.methods.split(",") if m],
                               settings=settings, workers=a.workers, seed=a.seed,
                               reward_factory=lambda b: SequenceLogProbabilityReward(b, coefficient=0.5))
    finally:
        backend.close()
    report.update(model=a.model, data="synthetic uniform-random prompts"
                  + (", random-init weights" if a.model.startswith("random:") else ""))
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(report, indent=2, default=str))
    print(json.dumps({"output": str(a.output), "speedup": {m: r["speedup"] for m, r in report["methods"].items()}}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
