"""dLLM infrastructure ablations: scheduling, resumption, streaming rewards, MH, IS and SMC arms.

Each family pairs two ways of doing the same diffusion work on one backend, prompt and seed
set, and records device / wall seconds, the generated tokens and the backend's counters
(forward calls, token slots) for each arm:

* ``block_continuous_batching`` -- four block requests one call at a time against one
  grouped call;
* ``resume_committed_blocks`` -- after an interruption that kept the first committed
  block, regenerating everything against continuing from the committed block;
* ``streaming_reward`` -- a slow reward (``--reward-delay`` seconds) computed after the
  batch one sequence at a time against on a thread pool;
* ``delayed_acceptance_mh`` -- reward MH against delayed-acceptance MH with a cheap
  surrogate reward (exact reward evaluations counted);
* ``progressive_is`` -- conditional IS against progressive IS at the same rollout budget;
* ``block_smc_rollout_forest`` -- the SMC rollout forest without and with reservoir reuse.

    python -m online_speculation_b200.experiments.dllm_infra --output dllm_infra.json \\
        [--config dllm.toml] [--families all] [--block-length 32] [--generation 64]

(without ``--config`` the backend holds random-init weights of the tiny MoE preset; a config's
``[model] path`` may name ``random:llada-moe-7b-a1b`` or a local LLaDA-MoE checkpoint.)

Families and arm names follow experiments/dllm/benchmark_infra.py; the GSM8K prompts and
verifier of that script are replaced by uniform-random prompts and a token-count reward.
"""

from __future__ import annotations

import argparse
import json
import time
from collections.abc import Callable, Sequence
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path
from typing import Any

import numpy as np

from ..dllm.config import DiffusionISConfig, DiffusionMHConfig, DiffusionSamplingConfig
from ..dllm.types import DiffusionGenerationRequest
from ..shared.config import SMCForestConfig
from ..shared.rng import SeedStream
from .rollout_infra import counter_delta, measure

FAMILIES = ("block_continuous_batching", "resume_committed_blocks", "streaming_reward", "delayed_acceptance_mh",
            "progressive_is", "block_smc_rollout_forest")


def _arm(backend, call: Callable[[], tuple[Sequence[int], dict]]) -> dict:
    snap = getattr(backend, "snapshot", lambda: None)
    before = snap()
    (tokens, info), t = measure(call)
    return {"telemetry": t, "tokens": len(tokens), "backend": counter_delta(before, snap()), **info}


def run_families(backend, *, prompt: tuple, sampling: DiffusionSamplingConfig, block: int, generation: int,
                 families: Sequence[str] = FAMILIES, seed: int = 20260812, reward_delay: float = 0.01,
                 candidates: int = 3, rollouts: int = 2) -> dict[str, dict[str, Any]]:
    """Every requested family's arms on one backend (``generation`` a multiple of ``block``)."""
    if generation % block or block % sampling.block_length:
        raise ValueError("the generation length is whole decision blocks of whole diffusion blocks")
    seeds = SeedStream(seed)
    unknown = set(families) - set(FAMILIES)
    if unknown:
        raise ValueError(f"unknown families: {sorted(unknown)}")

    def req(prefix, length, *path):
        return DiffusionGenerationRequest(tuple(prefix), length, sampling, seeds.derive("infra", *path),
                                          "infra:" + ":".join(str(p) for p in path))

    def count_reward(_p, y):
        return float(sum(int(t) % 2 for t in y)) / max(1, len(y))

    def batch_reward(p, ys):
        return [count_reward(p, y) for y in ys]

    out: dict[str, dict[str, Any]] = {}
    if "block_continuous_batching" in families:
        reqs = [req(prompt, block, "batch", i) for i in range(4)]

        def sequential():
            s = [backend.sample_batch((r,))[0] for r in reqs]
            return [t for x in s for t in x.token_ids], {"requests": 4, "calls": 4}

        def batched():
            s = backend.sample_batch(reqs)
            return [t for x in s for t in x.token_ids], {"requests": 4, "calls": 1}

        out["block_continuous_batching"] = {"sequential": _arm(backend, sequential), "batched": _arm(backend, batched)}
    if "resume_committed_blocks" in families:
        n_blocks = generation // block

        def blocks(resume: bool):
            first = backend.sample_batch((req(prompt, block, "resume", 0),))[0].token_ids
            done = tuple(first) if resume else ()
            for k in range(1 if resume else 0, n_blocks):
                done += tuple(backend.sample_batch((req(tuple(prompt) + done, block, "resume", k),))[0].token_ids)
            return done, {"committed_blocks_kept": 1 if resume else 0}

        out["resume_committed_blocks"] = {"restart_after_interruption": _arm(backend, lambda: blocks(False)),
                                          "resume_committed": _arm(backend, lambda: blocks(True))}
    if "streaming_reward" in families:
        reqs = [req(prompt, block, "stream", i) for i in range(4)]

        def slow(y):
            time.sleep(reward_delay)
            return count_reward(prompt, y)

        def serial():
            s = backend.sample_batch(reqs)
            return [t for x in s for t in x.token_ids], {"rewards": [slow(x.token_ids) for x in s]}

        def pooled():
            s = backend.sample_batch(reqs)
            with ThreadPoolExecutor(max_workers=4) as pool:
                r = list(pool.map(lambda x: slow(x.token_ids), s))
            return [t for x in s for t in x.token_ids], {"rewards": r}

        out["streaming_reward"] = {"after_batch": _arm(backend, serial), "thread_pool": _arm(backend, pooled)}
    if "delayed_acceptance_mh" in families:
        from ..dllm.algorithms import run_diffusion_reward_mh, run_diffusion_reward_mh_delayed

        cfg = DiffusionMHConfig(total_length=generation, updates=6, reward_temperature=0.5)
        calls = {"exact": 0}

        def exact(p, y):
            calls["exact"] += 1
            return count_reward(p, y)

        def standard():
            calls["exact"] = 0
            r = run_diffusion_reward_mh(backend=backend, prompt=prompt, config=cfg, sampling=sampling, reward=exact,
                                        seed=seed)
            return r.final.token_ids, {"exact_reward_evaluations": calls["exact"],
                                       "acceptance_rate": r.acceptance_rate}

        def delayed():
            calls["exact"] = 0
            r = run_diffusion_reward_mh_delayed(backend=backend, prompt=prompt, config=cfg, sampling=sampling,
                                                reward=exact, surrogate_reward=lambda p, y: 0.0, seed=seed)
            return r.final.token_ids, {"exact_reward_evaluations": calls["exact"],
                                       "surrogate_reward_evaluations": r.surrogate_reward_evaluations}

        out["delayed_acceptance_mh"] = {"reward_mh": _arm(backend, standard), "delayed_acceptance": _arm(backend, delayed)}
    if "progressive_is" in families:
        from ..dllm.algorithms import run_conditional_diffusion_is, run_progressive_diffusion_is

        cfg = DiffusionISConfig(candidate_count=candidates, rollout_count=rollouts, block_size=block,
                                total_length=generation, reward_temperature=0.5)

        def conditional():
            r = run_conditional_diffusion_is(base_backend=backend, prompt=prompt, config=cfg, base_sampling=sampling,
                                             reward_batch=batch_reward, seed=seed)
            return r.token_ids, {"rollouts_per_decision": candidates * rollouts}

        def progressive():
            r = run_progressive_diffusion_is(backend=backend, prompt=prompt, config=cfg, sampling=sampling,
                                             reward_batch=batch_reward, pilot_rollouts_per_candidate=1,
                                             evaluation_rollout_budget=candidates * rollouts)
            return r.token_ids, {"rollouts_per_decision": candidates * rollouts}

        out["progressive_is"] = {"conditional_is": _arm(backend, conditional),
                                 "progressive_is": _arm(backend, progressive)}
    if "block_smc_rollout_forest" in families:
        from ..dllm.algorithms import run_diffusion_smc_rollout_forest

        def smc(reuse: bool):
            r = run_diffusion_smc_rollout_forest(backend=backend, prompt=prompt, config=SMCForestConfig(
                particle_count=candidates, branch_factor=2, rollout_count=rollouts, block_size=block,
                total_length=generation, reward_temperature=0.5, reuse_rollout_forest=reuse), sampling=sampling,
                reward_batch=batch_reward, seed=seed)
            return r.token_ids, {"fresh_rollouts": r.fresh_rollouts, "reused_rollouts": r.reused_rollouts}

        out["block_smc_rollout_forest"] = {"no_reuse": _arm(backend, lambda: smc(False)),
                                           "reuse": _arm(backend, lambda: smc(True))}
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.dllm_infra")
    p.add_argument("--output", type=Path, required=True)
    p.add_argument("--config", type=Path, help="TOML with [model] path / mask_token_id and [runtime] (dllm loader)")
    p.add_argument("--families", default="all", help="comma-separated families or 'all'")
    p.add_argument("--prompt-tokens", type=int, default=64)
    p.add_argument("--block-length", type=int, default=32, help="diffusion block (tokens)")
    p.add_argument("--steps-per-block", type=int, default=32)
    p.add_argument("--decision-block", type=int, default=32)
    p.add_argument("--generation", type=int, default=64)
    p.add_argument("--reward-delay", type=float, default=0.01)
    p.add_argument("--seed", type=int, default=20260812)
    a = p.parse_args(argv)
    import tomllib

    from ..dllm.loader import load_diffusion_backend

    config = tomllib.loads(a.config.read_text()) if a.config else {"model": {"path": "random:tiny-moe"}}
    backend = load_diffusion_backend(config, "base")
    vocab = int(backend.model.cfg.vocab_size) if hasattr(backend.model, "cfg") else 1024
    rng = np.random.default_rng(a.seed)
    prompt = tuple(int(t) for t in rng.integers(0, vocab - 1, a.prompt_tokens) if int(t) != backend.mask_token_id)
    sampling = DiffusionSamplingConfig(block_length=a.block_length, steps_per_block=a.steps_per_block,
                                       temperature=1.0, remasking="random", mask_token_id=backend.mask_token_id)
    fams = FAMILIES if a.families == "all" else tuple(a.families.split(","))
    report = {"workload": {"prompt_tokens": len(prompt), "block_length": a.block_length,
                           "steps_per_block": a.steps_per_block, "decision_block": a.decision_block,
                           "generation": a.generation, "seed": a.seed, "model": config["model"]["path"]},
              "families": run_families(backend, prompt=prompt, sampling=sampling, block=a.decision_block,
                                       generation=a.generation, families=fams, seed=a.seed,
                                       reward_delay=a.reward_delay)}
    a.output.parent.mkdir(parents=True, exist_ok=True)
    a.output.write_text(json.dumps(report, indent=2, default=float))
    print(json.dumps({"output": str(a.output), "seconds": {
        f"{fam}/{arm}": round(v["telemetry"]["device_seconds"], 3)
        for fam, arms in report["families"].items() for arm, v in arms.items()}}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
