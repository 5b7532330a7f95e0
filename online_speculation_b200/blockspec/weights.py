"""HF <-> dual-view weight bridge and the own ``blockspec-dual-view-v1`` checkpoint.

The public key map (own key -> HF key; draft tensors carry the ``_diff``
suffix, e.g. ``model.layers.0.self_attn.q_proj_diff.weight``), the AR-only Qwen3
import that copies the AR projections into the draft view, and the checkpoint
payload keys (format, config, state, trainable, optimizer, step, metadata,
source, training_state) are kept identical to
online-speculation/src/blockspec/parallel/weights.py:28-193 so that weights and
checkpoints move between the two projects.
"""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from .model import DualViewConfig, DualViewDecoder

FORMAT = "blockspec-dual-view-v1"


def file_sha256(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as f:
        for chunk in iter(lambda: f.read(8 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def source_identity(source) -> dict:
    if not isinstance(source, dict):
        raise ValueError("checkpoint source metadata must be a mapping")
    return {k: v for k, v in source.items() if k in ("weight_sha256", "config_sha256")}


def public_key_map(config: DualViewConfig, *, include_draft: bool = True) -> dict[str, str]:
    m = {"embedding.weight": "model.embed_tokens.weight", "norm.weight": "model.norm.weight"}
    if not config.tie_word_embeddings:
        m["head.weight"] = "lm_head.weight"
    for i in range(config.num_hidden_layers):
        own, src = f"layers.{i}.", f"model.layers.{i}."
        m[own + "input_norm.weight"] = src + "input_layernorm.weight"
        m[own + "post_norm.weight"] = src + "post_attention_layernorm.weight"
        for n in ("gate", "up", "down"):
            m[own + f"{n}.weight"] = src + f"mlp.{n}_proj.weight"
        for view, suffix in ((("ar", ""), ("draft", "_diff")) if include_draft else (("ar", ""),)):
            for n in ("q", "k", "v", "o"):
                for kind in (("weight", "bias") if config.attention_bias else ("weight",)):
                    m[own + f"attention.{view}.{n}.{kind}"] = src + f"self_attn.{n}_proj{suffix}.{kind}"
            for n in ("q_norm", "k_norm"):
                m[own + f"attention.{view}.{n}.weight"] = src + f"self_attn.{n}{suffix}.weight"
    return m


def _finish(model: DualViewDecoder, state: dict, source: dict) -> DualViewDecoder:
    if model.config.tie_word_embeddings:
        state["head.weight"] = state["embedding.weight"]
    model.load_state_dict(state, strict=True, assign=True)
    model.tie_weights()
    model.frequencies = model._frequencies(model.embedding.weight.device)
    model.source = source
    return model.eval().requires_grad_(False)


def _read_safetensors(path: Path) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    from safetensors.torch import load_file

    index = path / "model.safetensors.index.json"
    files = sorted(set(json.loads(index.read_text())["weight_map"].values())) if index.exists() else ["model.safetensors"]
    tensors, digests = {}, {}
    for name in files:
        f = (path / name).resolve()
        if f.parent != path.resolve() or f.suffix != ".safetensors":
            raise ValueError("checkpoint shards must be local safetensors files")
        digests[name] = file_sha256(f)
        for k, v in load_file(str(f)).items():
            if k in tensors:
                raise ValueError(f"duplicate tensor {k}")
            tensors[k] = v
    return tensors, digests


def load_ar_base(path, *, block_size: int, mask_token_id: int, device="cpu") -> DualViewDecoder:
    """Plain Qwen3 AR checkpoint -> dual-view model whose draft view starts as a copy of AR."""
    path = Path(path)
    data = json.loads((path / "config.json").read_text())
    if data.get("model_type") != "qwen3":
        raise ValueError("a plain Qwen3 AR checkpoint is required")
    config = DualViewConfig.from_public(data | {"block_size": block_size, "mask_token_id": mask_token_id})
    mapping = public_key_map(config, include_draft=False)
    tensors, digests = _read_safetensors(path)
    if config.tie_word_embeddings and "lm_head.weight" in tensors:
        if not torch.equal(tensors.pop("lm_head.weight"), tensors["model.embed_tokens.weight"]):
            raise ValueError("tied AR output head differs from embeddings")
    if set(tensors) != set(mapping.values()):
        raise ValueError(f"AR tensors differ: missing={set(mapping.values()) - set(tensors)}, "
                         f"unexpected={set(tensors) - set(mapping.values())}")
    state = {own: tensors[src].to(device=device, dtype=torch.float32) for own, src in mapping.items()}
    for own in public_key_map(config):
        if ".attention.draft." in own:
            state[own] = state[own.replace(".attention.draft.", ".attention.ar.")].clone()
    with torch.device("meta"):
        model = DualViewDecoder(config)
    return _finish(model, state, {"kind": "ar-initialization", "config_sha256": file_sha256(path / "config.json"),
                                  "weight_sha256": digests})


def load_public(path, *, device="cpu", dtype=torch.float32, expected_sha256: str | None = None) -> DualViewDecoder:
    """Published dual-view checkpoint (HF names, ``_diff`` draft tensors)."""
    path = Path(path)
    config = DualViewConfig.from_public(json.loads((path / "config.json").read_text()))
    tensors, digests = _read_safetensors(path)
    digest = digests.get("model.safetensors")
    if expected_sha256 is not None and digest != expected_sha256:
        raise ValueError("public weight SHA256 mismatch")
    mapping = public_key_map(config)
    if config.tie_word_embeddings and "lm_head.weight" in tensors:
        if not torch.equal(tensors.pop("lm_head.weight"), tensors["model.embed_tokens.weight"]):
            raise ValueError("tied output head differs from token embeddings")
    if set(tensors) != set(mapping.values()):
        raise ValueError("public tensor keys differ")
    with torch.device("meta"):
        model = DualViewDecoder(config)
    expected = model.state_dict()
    state = {}
    for own, src in mapping.items():
        t = tensors[src]
        if t.shape != expected[own].shape:
            raise ValueError(f"shape mismatch for {src}")
        state[own] = t.to(device=device, dtype=dtype)
    return _finish(model, state, {"weight_sha256": digest, "config_sha256": file_sha256(path / "config.json")})


def export_public(model: DualViewDecoder, path) -> None:
    """Write the HF-named dual-view checkpoint (config.json + model.safetensors)."""
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    c = model.config
    sd = model.state_dict()
    save_file({src: sd[own].detach().contiguous().cpu() for own, src in public_key_map(c).items()},
              str(path / "model.safetensors"))
    data = {"model_type": "qwen3", "hidden_act": "silu", **{k: v for k, v in c.to_dict().items()},
            "rope_parameters": {"rope_type": "default", "rope_theta": c.rope_theta}}
    (path / "config.json").write_text(json.dumps(data, indent=1))


def save_checkpoint(path, model: DualViewDecoder, *, optimizer=None, step=0, metadata=None, training_state=None):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    payload = {"format": FORMAT, "config": model.config.to_dict(),
               "state": {k: v.detach().cpu() for k, v in model.state_dict().items()},
               "trainable": [n for n, p in model.named_parameters() if p.requires_grad],
               "optimizer": None if optimizer is None else optimizer.state_dict(),
               "step": step, "metadata": metadata or {}, "source": source_identity(getattr(model, "source", {})),
               "training_state": training_state}
    with path.open("xb") as f:
        torch.save(payload, f)


def load_checkpoint(path, *, device="cpu"):
    payload = torch.load(path, map_location=device, weights_only=True)
    if payload.get("format") != FORMAT:
        raise ValueError("unknown dual-view checkpoint format")
    config = DualViewConfig(**payload["config"])
    with torch.device("meta"):
        model = DualViewDecoder(config)
    expected, state = model.state_dict(), payload["state"]
    if set(expected) != set(state):
        raise ValueError("checkpoint tensor keys differ")
    for k, v in state.items():
        if v.shape != expected[k].shape or not torch.isfinite(v).all():
            raise ValueError(f"invalid checkpoint tensor: {k}")
    if config.tie_word_embeddings and not torch.equal(state["embedding.weight"], state["head.weight"]):
        raise ValueError("checkpoint tied weights differ")
    model = _finish(model, dict(state), source_identity(payload["source"]))
    params = dict(model.named_parameters())
    if set(payload["trainable"]) - params.keys():
        raise ValueError("unknown trainable checkpoint parameters")
    for n in payload["trainable"]:
        params[n].requires_grad_(True)
    return model, {k: payload.get(k) for k in ("optimizer", "step", "metadata", "training_state")}
