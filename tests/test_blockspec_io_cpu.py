"""Local tokenizer and the pinned-reference integrity gate (CPU)."""

import hashlib
import json

import pytest

from online_speculation_b200.blockspec.reference import checked_reference
from online_speculation_b200.blockspec.tokenizer import LocalTokenizer


def _write_tokenizer(directory, template=True):
    from tokenizers import Tokenizer, models, pre_tokenizers

    vocab = {"<unk>": 0, "<s>": 1, "</s>": 2, "hello": 3, "world": 4, "user": 5, ":": 6}
    tok = Tokenizer(models.WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = pre_tokenizers.Whitespace()
    tok.save(str(directory / "tokenizer.json"))
    config = {"bos_token": {"content": "<s>"}, "eos_token": "</s>"}
    if template:
        config["chat_template"] = ("{% for m in messages %}{{ m['role'] }}: {{ m['content'] }}\n{% endfor %}"
                                   "{% if add_generation_prompt %}assistant:{% endif %}")
    (directory / "tokenizer_config.json").write_text(json.dumps(config))


def test_local_tokenizer_round_trip_and_template(tmp_path):
    _write_tokenizer(tmp_path)
    tok = LocalTokenizer(tmp_path)
    ids = tok.encode("hello world")
    assert ids == [3, 4] and tok.decode(ids) == "hello world"
    text = tok.render_chat([{"role": "user", "content": "hello"}], add_generation_prompt=True)
    assert text == "user: hello\nassistant:"
    (tmp_path / "chat_template.jinja").write_text("{{ messages[0]['content'] }}!")
    assert LocalTokenizer(tmp_path).render_chat([{"role": "user", "content": "hi"}]) == "hi!"


def test_local_tokenizer_refuses_an_implicit_template(tmp_path):
    _write_tokenizer(tmp_path, template=False)
    with pytest.raises(ValueError, match="no local chat template"):
        LocalTokenizer(tmp_path).render_chat([{"role": "user", "content": "hello"}])


def _pinned(tmp_path):
    model = tmp_path / "model"
    model.mkdir()
    (model / "modeling.py").write_bytes(b"x = 1\r\ny = 2\r\n")
    (model / "config.json").write_text('{"a": 1}\n')
    (model / "model.safetensors").write_bytes(b"\x00\x01" * 1000)
    lf = {name: hashlib.sha256((model / name).read_bytes().replace(b"\r\n", b"\n")).hexdigest()
          for name in ("modeling.py", "config.json")}
    spec = {"reference_lf_sha256": lf, "weight_filename": "model.safetensors",
            "weight_sha256": hashlib.sha256((model / "model.safetensors").read_bytes()).hexdigest()}
    manifest = tmp_path / "manifest.json"
    manifest.write_text(json.dumps({"models": {"base": spec}}))
    return model, manifest, spec


def test_reference_gate_accepts_pins_and_refuses_changes(tmp_path):
    model, manifest, spec = _pinned(tmp_path)
    assert checked_reference(model, manifest) == spec
    (model / "modeling.py").write_bytes(b"x = 1\ny = 2\n")                 # LF-normalised: same digest
    assert checked_reference(model, manifest) == spec
    (model / "modeling.py").write_bytes(b"x = 3\n")
    with pytest.raises(ValueError, match="modeling.py"):
        checked_reference(model, manifest)


def test_reference_gate_refuses_escapes_weights_and_foreign_shards(tmp_path):
    model, manifest, spec = _pinned(tmp_path)
    (model / "model.safetensors.index.json").write_text(json.dumps({"weight_map": {"w": "other.safetensors"}}))
    with pytest.raises(ValueError, match="index"):
        checked_reference(model, manifest)
    (model / "model.safetensors.index.json").unlink()
    (model / "model.safetensors").write_bytes(b"\x00")
    with pytest.raises(ValueError, match="model.safetensors"):
        checked_reference(model, manifest)
    escape = dict(spec, reference_lf_sha256={"../manifest.json": "0" * 64})
    manifest.write_text(json.dumps({"models": {"base": escape}}))
    with pytest.raises(ValueError, match="not directly inside"):
        checked_reference(model, manifest)
