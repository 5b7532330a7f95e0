"""CPU tests of the AR / dLLM experiment pairing check."""

import pytest

from online_speculation_b200.experiments.pairing import SECTIONS, check_pairing, load_pairing


def _complete():
    cfg = {s: [{"ar": n, "dllm": f"d_{n}", **({"relation": "matched_role"} if s == "main_pairs" else {})}
               for n in sorted(names)] for s, names in SECTIONS.items()}
    cfg.update(run={"sample_count": 32}, passk={"draws": 8}, model={"architecture": "masked_diffusion_moe"})
    return cfg


def test_complete_pairing_passes_and_loads(tmp_path):
    out = check_pairing(_complete())
    assert set(out) == set(SECTIONS) and all(len(out[s]) == len(SECTIONS[s]) for s in SECTIONS)
    lines = ["[run]", "sample_count = 32", "[passk]", "draws = 8", "[model]", 'architecture = "masked_diffusion_moe"']
    for s, names in SECTIONS.items():
        for n in sorted(names):
            lines += [f"[[{s}]]", f'ar = "{n}"', f'dllm = "d_{n}"'] + (['relation = "exact_rule"'] if s == "main_pairs"
                                                                       else [])
    f = tmp_path / "pairing.toml"
    f.write_text("\n".join(lines) + "\n")
    _, sections = load_pairing(f)
    assert sections["training_pairs"][0].ar == "grpo"


@pytest.mark.parametrize("breakage", ["missing", "duplicate", "empty", "relation", "split", "draws", "arch"])
def test_broken_pairings_are_refused(breakage):
    cfg = _complete()
    if breakage == "missing":
        cfg["replay_pairs"] = cfg["replay_pairs"][:1]
    elif breakage == "duplicate":
        cfg["infra_pairs"].append(dict(cfg["infra_pairs"][0]))
    elif breakage == "empty":
        cfg["dynamic_pairs"][0]["dllm"] = ""
    elif breakage == "relation":
        cfg["main_pairs"][0]["relation"] = "vibes"
    elif breakage == "split":
        cfg["run"]["sample_count"] = 16
    elif breakage == "draws":
        cfg["passk"]["draws"] = 4
    else:
        cfg["model"]["architecture"] = "dense"
    with pytest.raises(ValueError):
        check_pairing(cfg)
