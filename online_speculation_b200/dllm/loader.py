"""Role-aware construction of masked-diffusion backends for paired experiments.

Config layout (the reference's, ``src/inference_scaling/dllm/backends/loader.py:13-70``)::

    [model]
    path = "inclusionAI/LLaDA-MoE-7B-A1B-Instruct"   # local HF checkpoint dir, or "random:<preset>"
    mask_token_id = 156895

    [runtime]
    device = "cuda"
    max_batch_size = 8

    [proposal]                     # role "proposal": early exit on the same resident weights
    kind = "shared_prefix_layers"
    layers = 8

    [alignment]                    # role "aligned": a VRPO adapter checkpoint (vrpo-lora-v1)
    adapter = "runs/vrpo/adapter.pt"

Roles: ``base`` (the full model), ``proposal`` (the first ``layers`` layers of the
base backend's weights), ``aligned`` (the base weights with the VRPO adapters
folded into the attention projections).
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from pathlib import Path
from typing import Any, Literal

import torch

from ..models.moe import PRESETS, MoEConfig, MoEDiffusionModel, build_weights, random_state_dict
from .backend import DiffusionEngineBackend

DiffusionRole = Literal["base", "proposal", "aligned"]


def config_from_hf(path: Path, mask_token_id: int | None = None) -> MoEConfig:
    """MoEConfig from a LLaDA-MoE ``config.json``."""
    c = json.loads((Path(path) / "config.json").read_text())
    return MoEConfig(
        vocab_size=int(c["vocab_size"]), hidden_size=int(c["hidden_size"]),
        num_hidden_layers=int(c["num_hidden_layers"]), num_attention_heads=int(c["num_attention_heads"]),
        num_key_value_heads=int(c.get("num_key_value_heads", c["num_attention_heads"])),
        head_dim=int(c.get("head_dim", c["hidden_size"] // c["num_attention_heads"])),
        num_experts=int(c["num_experts"]), num_experts_per_tok=int(c["num_experts_per_tok"]),
        moe_intermediate_size=int(c["moe_intermediate_size"]), norm_topk_prob=bool(c.get("norm_topk_prob", False)),
        rope_theta=float(c.get("rope_theta", 50000.0)), rms_norm_eps=float(c.get("rms_norm_eps", 1e-6)),
        qk_norm=bool(c.get("qk_layernorm", c.get("use_qk_norm", True))),
        tie_word_embeddings=bool(c.get("tie_word_embeddings", False)),
        mask_token_id=int(mask_token_id if mask_token_id is not None else c.get("mask_token_id", 156895)),
        name=Path(path).name)


def load_weights(path: str, *, device="cuda", mask_token_id: int | None = None, seed: int = 0):
    if path.startswith("random:"):
        cfg = PRESETS[path.split(":", 1)[1]]
        return build_weights(cfg, random_state_dict(cfg, seed=seed, device=device), device=device)
    from ..arllm.backends.loader import load_state_dict

    cfg = config_from_hf(Path(path), mask_token_id)
    return build_weights(cfg, load_state_dict(Path(path), device=device), device=device)


def load_diffusion_backend(config: Mapping[str, Any], role: DiffusionRole, *,
                           base_backend: DiffusionEngineBackend | None = None) -> DiffusionEngineBackend:
    model = dict(config["model"])
    runtime = dict(config.get("runtime", {}))
    path = str(model["path"])
    device = str(runtime.get("device", "cuda"))
    mask = model.get("mask_token_id")
    max_batch = int(runtime.get("max_batch_size", 8))
    if role not in ("base", "proposal", "aligned"):
        raise ValueError(f"unknown diffusion role {role!r}")

    def base():
        w = load_weights(path, device=device, mask_token_id=mask, seed=int(runtime.get("seed", 0)))
        return DiffusionEngineBackend(MoEDiffusionModel(w), model_id=path, mask_token_id=w.config.mask_token_id,
                                      max_batch_size=max_batch)

    if role == "base":
        return base()
    if role == "proposal":
        prop = dict(config["proposal"])
        if str(prop.get("kind")) != "shared_prefix_layers":
            raise ValueError("only the shared prefix-layer proposal is supported")
        layers = int(prop["layers"])
        if layers <= 0:
            raise ValueError("proposal.layers must be positive")
        return (base_backend or base()).with_prefix_layers(layers)
    adapter = Path(str(config["alignment"]["adapter"]))
    if not adapter.is_file():
        raise FileNotFoundError(f"aligned adapter is absent: {adapter}; run the VRPO stage first")
    from ..training.lora import LoRAConfig
    from ..training.vrpo import FORMAT, LoRAMoEPolicy

    st = torch.load(adapter, map_location="cpu", weights_only=False)
    if st.get("format") != FORMAT:
        raise ValueError("not a VRPO adapter checkpoint")
    w = load_weights(path, device=device, mask_token_id=mask, seed=int(runtime.get("seed", 0)))
    pol = LoRAMoEPolicy(w, LoRAConfig(**st["lora"]))
    if pol.flat.numel() != st["adapters"].numel():
        raise ValueError("adapter checkpoint does not match the model's LoRA layout")
    with torch.no_grad():
        pol.flat.copy_(st["adapters"].to(pol.flat.device))
    merged = pol.merged_weights()
    return DiffusionEngineBackend(MoEDiffusionModel(merged), model_id=str(adapter),
                                  mask_token_id=merged.config.mask_token_id, max_batch_size=max_batch)


__all__ = ["DiffusionRole", "config_from_hf", "load_diffusion_backend", "load_weights"]
