"""CPU tests of the report scrubber, the same-prefix draft audit and prompt rendering
(reference: online-speculation/src/blockspec/reporting.py, parallel/audit.py and
src/inference_scaling/shared/prompting.py)."""

import json
import math
import os
import socket

import pytest
import torch

from online_speculation_b200.blockspec.audit import audit
from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder
from online_speculation_b200.blockspec.reporting import parameter_digest, scrub, write_report
from online_speculation_b200.shared.prompting import render_prompt

CFG = DualViewConfig(vocab_size=17, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=4, block_size=4, mask_token_id=1)


def test_scrub_drops_identities_and_non_finite_numbers(tmp_path):
    home = os.path.expanduser("~")
    payload = {"checkpoint_path": "/data/model", "output_dirs": ["/a", "/b"], "actual_path": 3.5,
               "note": f"{home}/runs on {socket.gethostname()}", "loss": math.nan, "series": [1.0, math.inf],
               "nested": {"hostname": "box", "value": 2}}
    out = scrub(payload)
    assert "checkpoint_path" not in out and "output_dirs" not in out and "hostname" not in out["nested"]
    assert out["actual_path"] == 3.5                      # a measurement under a location-like key stays
    assert out["note"] == "~/runs on <host>" and out["loss"] is None and out["series"] == [1.0, None]
    f = tmp_path / "r.json"
    write_report(f, payload)
    assert json.loads(f.read_text()) == out and not (tmp_path / "r.json.tmp").exists()


def test_parameter_digest_tracks_weights():
    torch.manual_seed(0)
    a = DualViewDecoder(CFG)
    d = parameter_digest(a)
    assert d == parameter_digest(a)
    with torch.no_grad():
        next(a.parameters()).add_(1e-3)
    assert parameter_digest(a) != d


def test_audit_is_zero_change_for_identical_models_and_detects_a_change():
    torch.manual_seed(1)
    original = DualViewDecoder(CFG).eval()
    learned = DualViewDecoder(CFG).eval()
    learned.load_state_dict(original.state_dict())
    seqs = torch.randint(2, 17, (3, 16))
    anchors = torch.tensor([[2, 7], [3, 9], [4, 8]])
    same = audit(original, learned, seqs, anchors)
    assert same["kl_change"] == pytest.approx(0.0, abs=1e-7) and same["tv_change"] == pytest.approx(0.0, abs=1e-7)
    assert same["original"]["kl"] >= 0 and 0 <= same["original"]["tv"] <= 1
    with torch.no_grad():
        for layer in learned.layers:
            layer.attention.draft.q.weight.add_(torch.randn_like(layer.attention.draft.q.weight))
    moved = audit(original, learned, seqs, anchors)
    assert moved["learned"]["tv"] != pytest.approx(moved["original"]["tv"])


class _Tok:
    def __init__(self, template):
        self.chat_template = template
        self.calls = []

    def apply_chat_template(self, messages, tokenize, add_generation_prompt, **kw):
        self.calls.append(kw)
        return "<chat>" + "|".join(m["content"] for m in messages) + f"<think={kw.get('enable_thinking')}>"


def test_render_prompt_formats():
    msgs = [{"role": "user", "content": "2+2?"}]
    assert render_prompt(_Tok(None), msgs, {}) == "2+2?"                     # auto without a template: plain
    two = [{"role": "system", "content": "be brief"}, {"role": "user", "content": "hi"}]
    assert render_prompt(_Tok(None), two, {"prompt": {"format": "plain"}}) == "system: be brief\n\nuser: hi\n\nassistant:"
    tok = _Tok("{% if enable_thinking %}...{% endif %}")
    out = render_prompt(tok, msgs, {"output": {"thinking_mode": "disabled"}})
    assert out == "<chat>2+2?<think=False>" and tok.calls[-1] == {"enable_thinking": False}
    with pytest.raises(ValueError):
        render_prompt(_Tok(None), msgs, {"prompt": {"format": "chat"}})
    with pytest.raises(ValueError):
        render_prompt(tok, msgs, {"prompt": {"format": "json"}})
    with pytest.raises(ValueError):
        render_prompt(tok, msgs, {"prompt": {"chat_template_kwargs": {"tokenize": True}}})
    with pytest.raises(ValueError):
        render_prompt(tok, msgs, {"prompt": {"chat_template_kwargs": {"enable_thinking": True}},
                                  "output": {"thinking_mode": "disabled"}})
