"""The frozen pairing of autoregressive and diffusion experiments: load, check and print it.

A pairing file (TOML) names, for every comparison section, which dLLM method or arm stands
opposite each AR method or arm::

    [[main_pairs]]
    ar = "conditional_is"
    dllm = "conditional_is"
    relation = "exact_rule"            # main pairs state how the two correspond

    [run]
    sample_count = 32                  # the retained main split
    [passk]
    draws = 8
    [model]
    architecture = "masked_diffusion_moe"

:func:`check_pairing` requires every section to cover exactly its registered AR set (the
method registry's quality, pass@k and distribution methods; the replay and dynamic-IS arms;
the ablation axes; the infrastructure families; GRPO for training), each AR entry once and
with a non-empty counterpart, a known relation on every main pair, and the protocol
constants.  Section names, pair fields, relations and the AR sets are those of
experiments/shared/paired_protocol.py, so the reference's pairing files validate here.

    python -m online_speculation_b200.experiments.pairing --config pairing.toml
"""

from __future__ import annotations

import argparse
import tomllib
from collections.abc import Mapping
from dataclasses import dataclass
from pathlib import Path
from typing import Any

from .methods import AR_DISTRIBUTION_METHODS, AR_IS_PASSK_METHODS, AR_PAIRED_METHODS, AR_PASSK_METHODS

RELATIONS = frozenset({"exact_rule", "matched_role", "adapted"})
ABLATION_AXES = frozenset({"candidate_count", "rollout_count", "guidance_steps", "mh_alpha", "mh_updates",
                           "importance_clip", "generation_length", "reward_source", "temperature"})
INFRA_FAMILIES = frozenset({"continuous_batching", "resume_partial_rollouts", "streaming_reward", "history_token_tree",
                            "mh_proposal_tree_prefetch", "delayed_acceptance_mh", "replay_mixture_mh",
                            "progressive_is", "smc_rollout_forest", "vllm_backend"})
SECTIONS: Mapping[str, frozenset] = {
    "main_pairs": frozenset(AR_PAIRED_METHODS),
    "passk_pairs": frozenset(AR_PASSK_METHODS) | frozenset(AR_IS_PASSK_METHODS),
    "distribution_pairs": frozenset(AR_DISTRIBUTION_METHODS),
    "replay_pairs": frozenset({"fresh_only", "warm_replay"}),
    "dynamic_pairs": frozenset({"base_candidate_fixed", "replay_aware_fixed", "replay_aware_optimal"}),
    "ablation_pairs": ABLATION_AXES,
    "infra_pairs": INFRA_FAMILIES,
    "training_pairs": frozenset({"grpo"}),
}
MAIN_SPLIT = 32
PASSK_DRAWS = 8
ARCHITECTURE = "masked_diffusion_moe"


@dataclass(frozen=True, slots=True)
class MethodPair:
    ar: str
    dllm: str
    relation: str | None = None
    comparison: str | None = None


def check_pairing(config: Mapping[str, Any]) -> dict[str, tuple[MethodPair, ...]]:
    """Every section's pairs, after checking coverage, uniqueness and the protocol constants."""
    out: dict[str, tuple[MethodPair, ...]] = {}
    problems: list[str] = []
    for section, expected in SECTIONS.items():
        entries = config.get(section, ())
        try:
            pairs = tuple(MethodPair(**dict(e)) for e in entries)
        except TypeError as err:
            raise ValueError(f"{section}: every pair is a table with ar, dllm and optional relation / comparison "
                             f"({err})") from None
        names = [p.ar for p in pairs]
        if len(set(names)) != len(names):
            problems.append(f"{section} names an AR entry twice")
        missing, extra = sorted(expected - set(names)), sorted(set(names) - expected)
        if missing or extra:
            problems.append(f"{section}: missing {missing}, unexpected {extra}")
        if any(not p.dllm for p in pairs):
            problems.append(f"{section} has a pair without a dLLM counterpart")
        out[section] = pairs
    relations = {p.relation for p in out["main_pairs"]}
    if None in relations:
        problems.append("every main pair states its relation")
    elif not relations <= RELATIONS:
        problems.append(f"main pairs use unknown relations {sorted(relations - RELATIONS)}")
    if int(config.get("run", {}).get("sample_count", 0)) != MAIN_SPLIT:
        problems.append(f"the paired quality protocol keeps the {MAIN_SPLIT}-problem main split")
    if int(config.get("passk", {}).get("draws", 0)) != PASSK_DRAWS:
        problems.append(f"the paired pass@k protocol keeps {PASSK_DRAWS} independent draws")
    if config.get("model", {}).get("architecture") != ARCHITECTURE:
        problems.append(f"the dLLM counterpart declares model.architecture = {ARCHITECTURE!r}")
    if problems:
        raise ValueError("invalid pairing: " + "; ".join(problems))
    return out


def load_pairing(path: str | Path) -> tuple[dict[str, Any], dict[str, tuple[MethodPair, ...]]]:
    config = tomllib.loads(Path(path).read_text(encoding="utf-8"))
    return config, check_pairing(config)


def main(argv=None) -> int:
    p = argparse.ArgumentParser(prog="python -m online_speculation_b200.experiments.pairing")
    p.add_argument("--config", type=Path, required=True)
    a = p.parse_args(argv)
    _, sections = load_pairing(a.config)
    for section, pairs in sections.items():
        print(f"[{section}]")
        for pair in pairs:
            print(f"{pair.ar} -> {pair.dllm}" + (f" ({pair.relation})" if pair.relation else ""))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
