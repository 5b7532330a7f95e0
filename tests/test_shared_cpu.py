"""Shared layer on CPU: verifier plugin, numeric / consensus evaluation, consilience, generation budget,
thinking segmentation (markers, JSON, XML), model identity, budget allocation."""

from fractions import Fraction

import pytest

from online_speculation_b200.shared.budget import allocate_fresh_rollout_budget
from online_speculation_b200.shared.consilience import confidence_windows
from online_speculation_b200.shared.evaluation import (consensus_index, extract_numeric_answer, gsm8k_prompt,
                                                       modal_answer)
from online_speculation_b200.shared.generation import context_limit, generation_config_for_prompt
from online_speculation_b200.shared.model_loading import model_identity, model_loading_options
from online_speculation_b200.shared.output import ThinkingFormat, ThinkingParser
from online_speculation_b200.shared.structured_output import UnifiedOutputParser
from online_speculation_b200.shared.verifier import (ConfiguredTrainingVerifierReward, TokenVerifierReward,
                                                     VerifierContext, VerifierSpec, build_verifier)


def test_numeric_extraction_order_and_forms():
    assert extract_numeric_answer("so 3 then #### 1,234") == 1234
    assert extract_numeric_answer(r"\boxed{3/4} later 9") == Fraction(3, 4)
    assert extract_numeric_answer("The final answer is 2.5 apples") == Fraction(5, 2)
    assert extract_numeric_answer("numbers 1 and 7") == 7
    assert extract_numeric_answer("no digits") is None
    assert gsm8k_prompt("Q?").startswith("Q?\n\nSolve the problem step by step.")


def test_verifier_constant_python_and_version():
    const = build_verifier(VerifierSpec.from_mapping({"provider": "constant", "value": 0.5, "name": "c"}),
                           context=VerifierContext("p"))
    assert const.score("p", "x") == 0.5
    assert const.version.startswith("c:") and len(const.version) == 2 + 16
    spec = VerifierSpec.from_mapping({"factory": "online_speculation_b200.shared.evaluation.numeric:"
                                                 "build_numeric_reference_verifier", "requires_reference": True,
                                      "options": {"incorrect_reward": -1.0}})
    with pytest.raises(ValueError):
        build_verifier(spec, context=VerifierContext("q"))
    v = build_verifier(spec, context=VerifierContext("q", reference="42"))
    assert v.score("q", "#### 42") == 1.0 and v.score("q", "#### 41") == -1.0
    tok = TokenVerifierReward(v, lambda ids: "".join(chr(48 + i) for i in ids))
    assert tok((1,), (4, 2)) == 1.0 and tok.batch((1,), [(4, 2), (1,)]) == (1.0, -1.0)
    for bad in ({"provider": "constant"}, {"provider": "python"}, {"factory": "x:y", "value": 1},
                {"provider": "constant", "value": 1, "unknown": 2}):
        with pytest.raises((ValueError, TypeError)):
            VerifierSpec.from_mapping(bad)


def test_training_reward_groups_by_prompt_and_reference():
    spec = VerifierSpec.from_mapping({"factory": "online_speculation_b200.shared.evaluation.numeric:"
                                                 "build_numeric_reference_verifier", "requires_reference": True})
    r = ConfiguredTrainingVerifierReward(spec)
    out = r(["a", "a", "b"], ["#### 1", "#### 2", [{"content": "#### 3"}]], reference=["1", "1", "3"],
            completion_ids=[[1], [2, 3], [4]])
    assert out == [1.0, 0.0, 1.0]
    snap = r.snapshot(num_generations=3)
    assert snap["generated_completion_tokens"] == 4 and snap["observed_mean_reward"] == pytest.approx(2 / 3)


def test_consensus_and_consilience():
    assert modal_answer([Fraction(2), Fraction(1), Fraction(2), Fraction(1), None]) == 1
    assert consensus_index(["#### 3", "#### 5", "#### 3"], [-2.0, -0.1, -1.0]) == 2
    w = confidence_windows([1.0] * 10 + [3.0] * 10, window_fraction=0.25, skip_fraction=0.1)
    assert (w.skipped, w.window, w.initial, w.final) == (2, 5, 1.0, 3.0) and w.score == 0.0


def test_generation_budget_clips_to_context():
    class Cfg:
        max_position_embeddings = 1000

    class Backend:
        config = Cfg()

    assert context_limit(Backend()) == 1000
    cfg, info = generation_config_for_prompt({"generation": {"max_new_tokens": 5000}, "mh": {"block_size": 900}},
                                             200, [Backend()])
    assert cfg["generation"]["max_new_tokens"] == 800 and cfg["mh"]["block_size"] == 800
    assert info["length_limited_by_context"]


def test_thinking_marker_segmentation():
    fmt = ThinkingFormat(end_token_ids=(9,), start_token_ids=(8,), name="think")
    p = ThinkingParser((fmt,), is_blank=lambda t: all(x == 0 for x in t))
    s = p.split((1,), (8, 5, 6, 9, 7, 7, 3), eos_token_id=3)
    assert s.status == "complete" and s.thinking_token_ids == (5, 6) and s.content_token_ids == (7, 7)
    assert s.ended_by_eos
    assert p.split((1,), (8, 5, 6)).status == "incomplete"
    assert p.split((1, 8, 0), (5, 9, 4)).thinking_token_ids == (5,)          # opening marker prefilled
    assert p.split((1, 8, 0, 9, 0), (5, 6)).status == "disabled"
    assert p.split((1,), (4, 4, 8, 5, 9)).status == "leading_content"


def test_structured_json_and_xml_segmentation():
    dec = lambda ids: "".join(chr(i) for i in ids)  # noqa: E731 - one token per character
    enc = lambda s: tuple(ord(c) for c in s)  # noqa: E731
    parser = UnifiedOutputParser(ThinkingParser(()), decode=dec)
    js = enc('{"thinking": "add them", "answer": "42"}')
    s = parser.split((), js)
    assert s.status == "complete" and dec(s.thinking_token_ids) == "add them" and s.content_text == "42"
    xm = enc("<thinking>ok go</thinking><answer>7</answer>")
    s = parser.split((), xm)
    assert dec(s.thinking_token_ids) == "ok go" and dec(s.content_token_ids) == "7"
    assert parser.split((), enc('{"thinking": 3}')).status == "non_text_thinking_field"
    assert parser.split((), enc('{"thinking": "a", "thinking": "b"}')).status == "malformed_json"


def test_model_identity_and_loading_options():
    assert model_identity("m", "a", revision="r", tokenizer="t") == "m+adapter:a;revision=r;tokenizer=t"
    opts = model_loading_options({"model_loading": {"cache_dir": "c", "proposal": {"revision": "x"}}}, "proposal")
    assert opts == {"cache_dir": "c", "revision": "x", "local_files_only": True, "trust_remote_code": False}
    with pytest.raises(ValueError):
        model_loading_options({"model_loading": {"bogus": 1}})


def test_fresh_budget_is_proportional_to_std():
    a = allocate_fresh_rollout_budget(outer_ratios=[1, 1], standard_deviations=[1.0, 3.0], costs=[1, 1],
                                      rollout_budget=10)
    assert [x.fresh_count for x in a] == [3, 7] and sum(x.estimated_cost for x in a) <= 10
