"""Distribution audit of the samplers against exactly enumerable targets (CPU, no model files).

    python -m online_speculation_b200.experiments.distribution_audit --out audit.json \\
        [--chains 2000] [--runs 200] [--seed 0]

Two oracles:

* ``power``: a prefix-dependent three-token model, sequences of length 3 after a
  one-token prompt; the power target p(y)^alpha / Z is enumerated over all 27
  sequences and compared with the final states of batched suffix-MH chains by
  total variation (with the TV expected from sampling noise alone, estimated by
  drawing the same number of exact samples);
* ``reward``: the positional toy (vocabulary 32, length 12, i.i.d. N(0, 1) logits
  per position, reward = fraction of token 0, tau = 0.5), whose tilted target
  factorises over positions; per-position marginals of token 0 from reward MH
  and conditional IS runs are compared with the exact marginals (max absolute
  deviation and its z-score, expected count of zeros).

The JSON written to ``--out`` holds every figure; the exit status is non-zero when
a check fails its threshold.  The audits mirror the purpose of
experiments/arllm/gsm8k_distribution_audit.py (sampler output against its target
law) on oracles that need no model or dataset.
"""

from __future__ import annotations

import argparse
import itertools
import json
import math
from pathlib import Path

import numpy as np

from ..arllm.algorithms.conditional_is import run_conditional_is
from ..arllm.algorithms.mh import run_mh_chains_batched, run_reward_mh_chain
from ..arllm.backends.tabular import TabularBackend
from ..arllm.config import ConditionalISConfig, MHConfig, RewardMHConfig, SamplingConfig
from ..shared.metrics import empirical_distribution, total_variation
from ..shared.rng import SeedStream
from .artifacts import write_json_atomic


def _three_token_model() -> TabularBackend:
    def row(prefix):
        h = (sum(prefix) * 7 + len(prefix) * 3) % 5
        weights = np.array([1.0 + h, 2.0, 0.5 + 0.5 * h])
        return weights / weights.sum()

    return TabularBackend(row, 3)


def _power_target(backend: TabularBackend, prompt: tuple, length: int, alpha: float) -> dict:
    log_mass = {}
    for seq in itertools.product(range(backend.vocab_size), repeat=length):
        ctx, lp = list(prompt), 0.0
        for t in seq:
            lp += math.log(backend.probabilities(tuple(ctx))[t])
            ctx.append(t)
        log_mass[seq] = alpha * lp
    top = max(log_mass.values())
    total = sum(math.exp(v - top) for v in log_mass.values())
    return {k: math.exp(v - top) / total for k, v in log_mass.items()}


def audit_power_mh(chains: int, seed: int, *, alpha: float = 2.0, length: int = 3, iterations: int = 6) -> dict:
    backend = _three_token_model()
    prompt = (1,)
    target = _power_target(backend, prompt, length, alpha)
    cfg = MHConfig(alpha=alpha, total_length=length, block_size=length, iterations=iterations)
    results = run_mh_chains_batched(backend, prompt, cfg, SamplingConfig(temperature=1 / alpha),
                                    [SeedStream(seed * 100_003 + s) for s in range(chains)],
                                    chain_ids=list(range(chains)))
    tv = total_variation(empirical_distribution(r.token_ids for r in results), target)
    # the TV that exact samples of the same size show (sampling noise floor)
    rng = np.random.default_rng(seed)
    keys = list(target)
    draws = rng.choice(len(keys), size=chains, p=np.array([target[k] for k in keys]))
    noise = total_variation(empirical_distribution(keys[i] for i in draws), target)
    return {"chains": chains, "alpha": alpha, "length": length, "iterations": iterations, "tv": tv,
            "tv_exact_samples": noise, "passed": tv < max(0.05, 3 * noise)}


def _positional_oracle(backend: TabularBackend, length: int, tau: float) -> np.ndarray:
    tilted = backend.position_probabilities.copy()
    tilted[:, 0] *= math.exp(1.0 / (length * tau))
    return tilted / tilted.sum(-1, keepdims=True)


def audit_reward_samplers(runs: int, seed: int, *, vocab: int = 32, length: int = 12, tau: float = 0.5) -> dict:
    backend = TabularBackend.per_position_logits(vocab, length, seed=3, prompt_length=2)
    prompt = (5, 6)

    def reward(_prompt, y):
        return sum(t == 0 for t in y) / len(y)

    oracle = _positional_oracle(backend, length, tau)[:, 0]
    out = {"vocab": vocab, "length": length, "tau": tau, "runs": runs,
           "oracle_zero_marginals": oracle.tolist(), "oracle_expected_zeros": float(oracle.sum()),
           "base_expected_zeros": float(backend.position_probabilities[:, 0].sum())}
    samplers = {
        "reward_mh": lambda s: run_reward_mh_chain(
            backend, prompt, RewardMHConfig(total_length=length, block_size=length, reward_temperature=tau,
                                            iterations=64), SamplingConfig(), reward, SeedStream(s), chain_id=0),
        "conditional_is": lambda s: run_conditional_is(
            base_backend=backend, prompt=prompt, config=ConditionalISConfig(
                candidate_count=8, rollout_count=4, block_size=4, total_length=length, reward_temperature=tau),
            seeds=SeedStream(s), reward=reward),
    }
    for name, run in samplers.items():
        zeros = np.array([[t == 0 for t in run(seed * 10_007 + s).token_ids] for s in range(runs)], dtype=np.float64)
        marginals = zeros.mean(0)
        se = np.sqrt(np.maximum(oracle * (1 - oracle), 1e-12) / runs)
        dev = np.abs(marginals - oracle)
        entry = {"zero_marginals": marginals.tolist(), "max_abs_deviation": float(dev.max()),
                 "max_z": float((dev / se).max()), "expected_zeros": float(zeros.sum(1).mean())}
        # reward MH targets pi_r exactly; finite-candidate conditional IS is approximately exact
        limit = 4.5 if name == "reward_mh" else 6.0
        entry["passed"] = entry["max_z"] < limit
        out[name] = entry
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.distribution_audit")
    p.add_argument("--out", required=True)
    p.add_argument("--chains", type=int, default=2000, help="suffix-MH chains for the power-target audit")
    p.add_argument("--runs", type=int, default=200, help="runs per sampler for the reward audit")
    p.add_argument("--seed", type=int, default=0)
    a = p.parse_args(argv)
    report = {"power_mh": audit_power_mh(a.chains, a.seed), "reward": audit_reward_samplers(a.runs, a.seed)}
    checks = [report["power_mh"]["passed"], report["reward"]["reward_mh"]["passed"],
              report["reward"]["conditional_is"]["passed"]]
    report["passed"] = all(checks)
    write_json_atomic(Path(a.out), report, indent=2)
    print(json.dumps({"out": a.out, "passed": report["passed"], "power_tv": report["power_mh"]["tv"]}))
    return 0 if report["passed"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
