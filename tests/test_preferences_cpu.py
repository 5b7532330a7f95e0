"""CPU tests of the resumable preference-pair builder (behaviour of
experiments/dllm/prepare_gsm8k_vrpo.py): pair selection per problem, skipped problems,
resume after an interruption, fingerprint refusal, and the token triples for VRPO."""

import json
from dataclasses import dataclass
from fractions import Fraction

import pytest

from online_speculation_b200.experiments.preferences import (PreferenceRun, build_preference_pairs,
                                                             load_preference_pairs, load_problem_file)
from online_speculation_b200.shared.evaluation.gsm8k import GSM8KProblem
from online_speculation_b200.shared.verifier import VerifierSpec

NUMERIC = VerifierSpec.from_mapping({"provider": "python", "name": "numeric",
                                     "factory": "online_speculation_b200.shared.evaluation.numeric:"
                                                "build_numeric_reference_verifier",
                                     "requires_reference": True})


@dataclass
class _Sample:
    token_ids: tuple


class _Backend:
    """Answers problem i with '#### i' on even draws and '#### -1' on odd ones (problem 3: always right)."""

    def __init__(self):
        self.calls = 0

    def sample_batch(self, reqs):
        self.calls += 1
        out = []
        for r in reqs:
            prob, draw = (int(x) for x in r["id"].split(":")[1:])
            good = draw % 2 == 0 or prob == 3
            out.append(_Sample(tuple(f"#### {prob if good else -1}".encode())))
        return out

    def snapshot(self):
        return {"sample_calls": self.calls}


def _problems(n=8):
    return tuple(GSM8KProblem(i, f"q{i}", f"so the answer is\n#### {i}", Fraction(i)) for i in range(n))


def _build(tmp_path, backend, run, **kw):
    return build_preference_pairs(backend, _problems(), run, NUMERIC, encode_prompt=lambda t: list(t.encode()),
                                  decode=lambda ids: bytes(ids).decode(),
                                  make_request=lambda prefix, seed, rid: {"prefix": prefix, "seed": seed, "id": rid},
                                  output=tmp_path / "pairs.jsonl", manifest=tmp_path / "manifest.json",
                                  effective={"model": "stub"}, log=lambda _m: None, **kw)


def test_pairs_skips_and_manifest(tmp_path):
    run = PreferenceRun(max_pairs=7, candidate_pool_size=8, num_generations=4, seed=0,
                        include_reference_completion=False)
    res = _build(tmp_path, _Backend(), run)
    recs = [json.loads(x) for x in (tmp_path / "pairs.jsonl").read_text().splitlines()]
    assert res["status"] == "complete" and res["preference_pairs"] == 7
    by = {r["problem_index"]: r for r in recs}
    assert by[3]["status"] == "skipped_equal_verifier_rewards"           # every draw right: no preference
    pair = next(r for r in recs if r["status"] == "pair")
    assert pair["chosen"].endswith(f"#### {pair['problem_index']}") and pair["rejected"].endswith("#### -1")
    assert pair["chosen_source"] == "candidate:0" and pair["rejected_source"] == "candidate:1"
    assert [c["correct"] for c in pair["candidates"]] == [True, False, True, False]
    assert json.loads((tmp_path / "manifest.json").read_text())["fingerprint"] == pair["fingerprint"]


def test_reference_completion_joins_and_shortfall_raises(tmp_path):
    run = PreferenceRun(max_pairs=8, candidate_pool_size=8, num_generations=2, seed=0)
    with pytest.raises(RuntimeError, match="fewer"):
        _build(tmp_path, _Backend(), run)
    recs = [json.loads(x) for x in (tmp_path / "pairs.jsonl").read_text().splitlines()]
    assert len(recs) == 8 and all(r["reference_completion_verifier_reward"] == 1.0 for r in recs)


def test_resume_and_fingerprint_refusal(tmp_path):
    run = PreferenceRun(max_pairs=3, candidate_pool_size=8, num_generations=2, seed=1,
                        include_reference_completion=False)
    b = _Backend()
    _build(tmp_path, b, run)
    first = (tmp_path / "pairs.jsonl").read_text().splitlines()
    # running the same run again resumes from its records: no problem is drawn twice
    b2 = _Backend()
    _build(tmp_path, b2, run)
    assert b2.calls == 0 and (tmp_path / "pairs.jsonl").read_text().splitlines() == first
    with pytest.raises(ValueError, match="fingerprint"):
        _build(tmp_path, _Backend(), PreferenceRun(max_pairs=3, candidate_pool_size=8, num_generations=4, seed=1,
                                                   include_reference_completion=False))
    triples = load_preference_pairs(tmp_path / "pairs.jsonl", lambda t: list(t.encode()))
    assert len(triples) == 3 and all(len(p) and len(c) and len(r) for p, c, r in triples)


def test_problem_file_and_run_validation(tmp_path):
    f = tmp_path / "p.jsonl"
    f.write_text('{"question": "1+1?", "answer": "two\\n#### 2"}\n{"question": "x", "answer": "#### 3.5"}\n')
    probs = load_problem_file(f, pinned=False)
    assert [p.gold_answer for p in probs] == [Fraction(2), Fraction(7, 2)]
    with pytest.raises(ValueError):
        load_problem_file(f, pinned=True)
    with pytest.raises(ValueError):
        PreferenceRun(max_pairs=5, candidate_pool_size=4, num_generations=2, seed=0)
    with pytest.raises(ValueError):
        PreferenceRun(max_pairs=1, candidate_pool_size=4, num_generations=0, seed=0)
