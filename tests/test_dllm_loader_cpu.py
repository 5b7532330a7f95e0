"""Role-aware masked-diffusion backend loader and adapter merging (CPU)."""

from dataclasses import asdict

import pytest
import torch

from online_speculation_b200.dllm.config import DiffusionSamplingConfig
from online_speculation_b200.dllm.loader import load_diffusion_backend, load_weights
from online_speculation_b200.dllm.types import DiffusionGenerationRequest
from online_speculation_b200.training.lora import LoRAConfig
from online_speculation_b200.training.vrpo import FORMAT, LoRAMoEPolicy

CFG = {"model": {"path": "random:tiny-moe"}, "runtime": {"device": "cpu", "max_batch_size": 4},
       "proposal": {"kind": "shared_prefix_layers", "layers": 1}}


def _req(seed=0):
    return DiffusionGenerationRequest((3, 4, 5, 6), 8, DiffusionSamplingConfig(block_length=4, steps_per_block=4,
                                                                            temperature=1.0), seed, f"r{seed}")


def test_base_and_prefix_layer_proposal():
    base = load_diffusion_backend(CFG, "base")
    out = base.sample_batch([_req()])[0]
    assert len(out.token_ids) == 8
    prop = load_diffusion_backend(CFG, "proposal", base_backend=base)
    assert prop.model is base.model and "prefix-layers=1" in prop.model_id
    assert len(prop.sample_batch([_req(1)])[0].token_ids) == 8
    with pytest.raises(ValueError):
        load_diffusion_backend(dict(CFG, proposal={"kind": "other", "layers": 1}), "proposal", base_backend=base)


def test_aligned_role_folds_the_adapters(tmp_path):
    w = load_weights("random:tiny-moe", device="cpu")
    pol = LoRAMoEPolicy(w, LoRAConfig(rank=2, alpha=4.0))
    with torch.no_grad():
        pol.flat.normal_(0, 0.05)
    path = tmp_path / "adapter.pt"
    torch.save({"format": FORMAT, "adapters": pol.flat.detach().clone(), "lora": asdict(pol.lora)}, path)
    merged = pol.merged_weights()
    a = pol.adapters[0]["qkv"]
    want = w.layers[0].w_qkv.float() + pol.lora.scale * ((a.B * a.block_mask) @ a.A)
    assert torch.allclose(merged.layers[0].w_qkv.float(), want, atol=1e-2)
    assert merged.layers[0].router is w.layers[0].router          # untouched tensors are shared
    aligned = load_diffusion_backend(dict(CFG, alignment={"adapter": str(path)}), "aligned")
    assert aligned.model_id == str(path)
    assert torch.allclose(aligned.model.w.layers[1].w_o.float(), merged.layers[1].w_o.float())
    assert len(aligned.sample_batch([_req(2)])[0].token_ids) == 8
    with pytest.raises(FileNotFoundError):
        load_diffusion_backend(dict(CFG, alignment={"adapter": str(tmp_path / "missing.pt")}), "aligned")
