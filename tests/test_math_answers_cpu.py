"""CPU tests of the MATH-style answer grading, the stratified subset and the isolated judge."""

import json

import pytest

from online_speculation_b200.shared.evaluation.math_answers import (MathJudge, answers_equivalent,
                                                                   build_math_reference_verifier, canonical_answer,
                                                                   final_answer, grade, load_math500,
                                                                   stratified_subset)
from online_speculation_b200.shared.verifier import VerifierContext, VerifierSpec, build_verifier


def test_final_answer_extraction():
    assert final_answer(r"so \boxed{\frac{1}{2}} and then \boxed{\dfrac{3}{4}}.") == r"\dfrac{3}{4}"
    assert final_answer(r"\boxed{\{1, 2\}}") == r"\{1, 2\}"
    assert final_answer(r"\boxed{x^{2}+\sqrt{3}}") == r"x^{2}+\sqrt{3}"
    assert final_answer("The answer is 42.") == "42"
    assert final_answer("no answer here") is None
    assert final_answer(r"\boxed{unclosed") is None


@pytest.mark.parametrize("a,b", [(r"\frac{1}{2}", "0.5"), (r"\dfrac12", "1/2"), ("3", "3.0"), ("1,000", "1000"),
                                 (r"\left(1,\frac{2}{4}\right)", "(1, 0.5)"), (r"90^\circ", "90"),
                                 (r"\text{(B)}", "(B)"), ("x=5", "5"), (r"\$12", "12"), ("50\\%", "50"),
                                 (r"2\sqrt{3}", r"2 \sqrt{3}"), ("[1,2)", "[1, 2)")])
def test_equivalent_spellings(a, b):
    assert answers_equivalent(a, b), (canonical_answer(a), canonical_answer(b))


@pytest.mark.parametrize("a,b", [("1/3", "0.33"), ("(1,2)", "(2,1)"), ("[1,2)", "(1,2)"), (r"\sqrt{2}", r"\sqrt{3}"),
                                 ("12", "13")])
def test_different_answers(a, b):
    assert not answers_equivalent(a, b)


def test_grade_and_verifier():
    assert grade(r"thus \boxed{\frac{3}{6}}", "1/2") == {"correct": True, "parseable": True, "reference_parseable": True}
    assert grade("nothing", "1/2")["parseable"] is False
    spec = VerifierSpec.from_mapping({"provider": "python", "name": "math",
                                      "factory": "online_speculation_b200.shared.evaluation.math_answers:"
                                                 "build_math_reference_verifier", "requires_reference": True})
    v = build_verifier(spec, context=VerifierContext(prompt="q", reference=r"\frac{1}{4}"))
    assert v.score("q", r"\boxed{0.25}") == 1.0 and v.score("q", r"\boxed{0.3}") == 0.0
    with pytest.raises(ValueError):
        build_math_reference_verifier(context=VerifierContext(prompt="q"))


def test_isolated_judge():
    judge = MathJudge(timeout_seconds=60)
    try:
        assert judge.grade(r"\boxed{2}", "2.0")["correct"]
        assert judge.equivalent("(1,2)", r"\left(1, 2\right)")
        with pytest.raises(ValueError):
            judge._call("unknown")
    finally:
        judge.close()


def test_stratified_subset(tmp_path):
    rows = [{"unique_id": f"p{i}", "problem": f"q{i}", "answer": str(i), "subject": ("alg", "geo", "num")[i % 3],
             "level": 1 + i % 5} for i in range(60)]
    f = tmp_path / "math.jsonl"
    f.write_text("\n".join(json.dumps(r) for r in rows))
    probs = load_math500(f)
    a = stratified_subset(probs, seed=3, minimum_level=2, development_count=4, test_count=10)
    b = stratified_subset(probs, seed=3, minimum_level=2, development_count=4, test_count=10)
    assert [p.identifier for p in a["test"]] == [p.identifier for p in b["test"]]
    chosen = a["development"] + a["test"]
    assert len({p.identifier for p in chosen}) == 14 and all(p.level >= 2 for p in chosen)
    # the first round visits every stratum once
    first = chosen[:12]
    assert len({(p.subject, p.level) for p in first}) == 12
    with pytest.raises(ValueError):
        stratified_subset(probs, seed=3, minimum_level=2, development_count=40, test_count=40)
    f.write_text("\n".join(json.dumps(r) for r in rows + rows[:1]))
    with pytest.raises(ValueError):
        load_math500(f)
