"""Token-gated low-rank decoder on CUDA: the drafting forward against the paired training layout,
exact greedy noise drafting, and one bf16-base / fp32-adapter distillation step."""

import pytest
import torch

from online_speculation_b200.blockspec.generation import generate, generate_ar
from online_speculation_b200.blockspec.lowrank import (LowRankConfig, LowRankDecoder, NoiseBranch, offline_step,
                                                       paired_batch)
from online_speculation_b200.blockspec.sampling import SamplingConfig

pytestmark = pytest.mark.gpu


def _model(dtype):
    torch.manual_seed(0)
    m = LowRankDecoder(LowRankConfig(vocab_size=96, hidden_size=64, head_dim=16, query_key_norm=True))
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("lora_B"):
                p.normal_(0, 0.3)
    return m.to("cuda", dtype).eval().requires_grad_(False)


def test_paired_layout_and_greedy_drafting_on_cuda():
    m = _model(torch.float64)
    K, L = 4, 16
    g = torch.Generator(device="cuda").manual_seed(1)
    clean = torch.randint(2, 96, (1, L), device="cuda", generator=g)
    noisy = torch.randint(2, 96, (1, L), device="cuda", generator=g)
    b = paired_batch(clean, K, noisy)
    paired = m(b.tokens, positions=b.positions, allowed=b.allowed, adapter_mask=b.adapter_mask).logits
    s = 8
    inputs = torch.cat((clean[:, s:s + 1], noisy[:, s + 1:s + K]), 1)
    route = torch.ones_like(inputs, dtype=torch.bool)
    route[:, 0] = False
    drafted = m(inputs, cache=m(clean[:, :s]).cache, adapter_mask=route).logits
    assert torch.allclose(drafted[:, 1:], paired[:, L + s + 1:L + s + K], atol=1e-9)
    br = NoiseBranch(m, block_size=4)
    prompt = torch.tensor([[5, 9, 13, 2, 7]], device="cuda")
    spec = generate(br, prompt, 40, sampling=SamplingConfig(0.0), generator=torch.Generator(device="cuda").manual_seed(0))
    assert spec.tokens == generate_ar(br, prompt, 40, sampling=SamplingConfig(0.0)).tokens


def test_bf16_base_distillation_step():
    m = _model(torch.float32).set_base_dtype(torch.bfloat16).train_adapters_only()
    assert all(p.dtype == torch.float32 for p in m.adapter_parameters())
    opt = torch.optim.Adam(m.adapter_parameters(), lr=1e-3)
    data = torch.randint(2, 96, (4, 32), device="cuda")
    rec = offline_step(m, opt, data, 4, generator=torch.Generator(device="cuda").manual_seed(0))
    assert torch.isfinite(torch.tensor(rec["loss"])) and rec["gradient_norm"] > 0


def test_cuda_graph_workspace_executor():
    from online_speculation_b200.blockspec.lowrank import NoiseBranch
    from online_speculation_b200.blockspec.lowrank_exec import GraphNoiseBranch

    m = _model(torch.float64)
    prompt = torch.tensor([[5, 9, 13, 2, 7, 1, 11, 4, 3, 8]], device="cuda")
    ws = GraphNoiseBranch(m, block_size=4, capacity=256)
    ws.prepare()
    eager = NoiseBranch(m, block_size=4)
    for t in (0.0, 1.0):
        s = SamplingConfig(t)
        a = generate(eager, prompt, 48, sampling=s, generator=torch.Generator(device="cuda").manual_seed(2))
        b = generate(ws, prompt, 48, sampling=s, generator=torch.Generator(device="cuda").manual_seed(2))
        assert a.tokens == b.tokens and a.accepted_per_round == b.accepted_per_round
    assert ws.graph_replays > 0 and ws.eager_forwards >= 1
