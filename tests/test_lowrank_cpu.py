"""Token-gated low-rank decoder and noise-input drafting (CPU): adapter gating, attention backends,
the paired training layout against the drafting forward, exact decoding, offline and online
adapter learning, checkpoints, and the Hugging Face import."""

import math

import pytest
import torch

from online_speculation_b200.blockspec.diffusion import UniformNoise
from online_speculation_b200.blockspec.generation import ProposalSampler, generate, generate_ar
from online_speculation_b200.blockspec.lowrank import (LowRankConfig, LowRankDecoder, LowRankFeedback,
                                                       LowRankLearner, NoiseBranch, from_hf, grouped_attention,
                                                       load, offline_step, paired_batch, paired_loss,
                                                       rotary_frequencies, save)
from online_speculation_b200.blockspec.sampling import SamplingConfig


def _model(seed=0, vocab=32, scale=0.3, **kw):
    torch.manual_seed(seed)
    m = LowRankDecoder(LowRankConfig(vocab_size=vocab, query_key_norm=True, **kw)).double().eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            if n.endswith("lora_B"):
                p.normal_(0, scale)
    return m.requires_grad_(False)


def test_adapter_gating():
    m = _model()
    x = torch.tensor([[3, 7, 1, 9, 4]])
    plain = m(x).logits
    off = m(x, adapter_mask=torch.zeros_like(x, dtype=torch.bool)).logits
    assert torch.equal(plain, off)
    route = torch.tensor([[False, False, True, True, False]])
    gated = m(x, adapter_mask=route).logits
    assert torch.allclose(gated[:, :2], plain[:, :2], atol=1e-12)     # rows before the first adapted row
    assert not torch.allclose(gated[:, 2:], plain[:, 2:])
    fresh = LowRankDecoder(LowRankConfig(vocab_size=32)).double()
    assert torch.allclose(fresh(x, adapter_mask=route).logits, fresh(x).logits)   # B starts at zero


def test_grouped_attention_matches_sdpa_and_empty_rows_are_zero():
    g = torch.Generator().manual_seed(1)
    q = torch.randn(2, 4, 3, 8, generator=g, dtype=torch.float64)
    k = torch.randn(2, 2, 7, 8, generator=g, dtype=torch.float64)
    v = torch.randn(2, 2, 7, 8, generator=g, dtype=torch.float64)
    allowed = torch.rand(1, 1, 3, 7, generator=g) < 0.6
    allowed[..., 0] = True
    want = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=allowed, enable_gqa=True)
    assert torch.allclose(grouped_attention(q, k, v, allowed), want, atol=1e-12)
    allowed[..., 1, :] = False
    assert torch.equal(grouped_attention(q, k, v, allowed)[:, :, 1], torch.zeros(2, 4, 8, dtype=torch.float64))
    m = _model(2)
    x = torch.tensor([[3, 7, 1, 9, 4, 2]])
    a = m(x, adapter_mask=x > 3).logits
    b = m.set_attention_backend("grouped")(x, adapter_mask=x > 3).logits
    assert torch.allclose(a, b, atol=1e-10)


def test_cache_and_suffix_recompute_match_the_full_forward():
    m = _model(3)
    x = torch.tensor([[3, 7, 1, 9, 4, 2, 8]])
    full = m(x, capture_layer=1)
    head = m(x[:, :4])
    tail = m(x[:, 4:], cache=head.cache).logits
    assert torch.allclose(tail, full.logits[:, 4:], atol=1e-10)
    assert torch.allclose(m.forward_suffix(full.boundary), full.logits, atol=1e-10)
    assert torch.allclose(m.forward_suffix(full.boundary, logit_range=(2, 5)), full.logits[:, 2:5], atol=1e-10)


def test_paired_layout_is_the_drafting_forward():
    m = _model(4)
    K, L = 4, 12
    g = torch.Generator().manual_seed(4)
    clean = torch.randint(2, 32, (1, L), generator=g)
    noisy = torch.randint(2, 32, (1, L), generator=g)
    b = paired_batch(clean, K, noisy)
    paired = m(b.tokens, positions=b.positions, allowed=b.allowed, adapter_mask=b.adapter_mask).logits
    assert torch.allclose(paired[:, :L], m(clean).logits, atol=1e-10)        # the teacher is the plain decoder
    for s in range(0, L, K):
        hist = None if s == 0 else m(clean[:, :s]).cache
        inputs = torch.cat((clean[:, s:s + 1], noisy[:, s + 1:s + K]), 1)
        route = torch.ones_like(inputs, dtype=torch.bool)
        route[:, 0] = False
        drafted = m(inputs, cache=hist, adapter_mask=route).logits
        assert torch.allclose(drafted[:, 1:], paired[:, L + s + 1:L + s + K], atol=1e-10)
    assert b.eligible.sum() == L - L // K


def test_yarn_ramp():
    plain = LowRankConfig(head_dim=64, rope_theta=1e6)
    yarn = LowRankConfig(head_dim=64, rope_theta=1e6, rope_factor=4.0, rope_original_length=4096)
    a, b = rotary_frequencies(plain), rotary_frequencies(yarn)
    assert torch.equal(a[:4], b[:4])                                          # fast dimensions keep their frequency
    assert torch.allclose(b[-2:], a[-2:] / 4)                                  # slow ones are interpolated
    assert bool((b <= a).all())
    m = LowRankDecoder(yarn).to(torch.bfloat16)
    assert m.frequencies.dtype == torch.float32


def test_greedy_noise_drafting_equals_ar():
    m = _model(5)
    br = NoiseBranch(m, block_size=4)
    prompt = torch.tensor([[5, 9, 13, 2, 7]])
    g = SamplingConfig(0.0)
    spec = generate(br, prompt, 30, sampling=g, generator=torch.Generator().manual_seed(0))
    assert spec.tokens == generate_ar(br, prompt, 30, sampling=g).tokens
    assert spec.rounds >= 1 and spec.decode_forwards < 30


def test_sampled_noise_drafting_follows_the_target_law():
    V = 5
    m = _model(6, vocab=V, scale=1.0)
    br = NoiseBranch(m, UniformNoise(0, V), block_size=3)
    prompt = torch.tensor([[3, 1]])
    with torch.no_grad():
        p1 = m(prompt).logits[0, -1].softmax(-1)
        exact = torch.zeros(V, V, dtype=torch.float64)
        for a in range(V):
            p2 = m(torch.tensor([[3, 1, a]])).logits[0, -1].softmax(-1)
            for b in range(V):
                p3 = m(torch.tensor([[3, 1, a, b]])).logits[0, -1].softmax(-1)
                exact[b] += p1[a] * p2[b] * p3
    g = torch.Generator().manual_seed(7)
    counts = torch.zeros(V, V, dtype=torch.float64)
    n = 1500
    for _ in range(n):
        out = generate(br, prompt, 3, sampling=SamplingConfig(1.0), generator=g)
        counts[out.tokens[1], out.tokens[2]] += 1
    assert 0.5 * float((counts / n - exact).abs().sum()) < 0.08


def test_offline_distillation_lowers_the_loss():
    torch.manual_seed(8)
    m = LowRankDecoder(LowRankConfig(vocab_size=24, adapter_rank=8)).train_adapters_only()
    data = torch.randint(2, 24, (8, 16))
    opt = torch.optim.Adam(m.adapter_parameters(), lr=1e-2)
    g = torch.Generator().manual_seed(0)
    with torch.no_grad():
        before = float(paired_loss(m, data, 4, generator=torch.Generator().manual_seed(1)))
    for _ in range(40):
        rec = offline_step(m, opt, data, 4, generator=g)
        assert math.isfinite(rec["loss"])
    with torch.no_grad():
        after = float(paired_loss(m, data, 4, generator=torch.Generator().manual_seed(1)))
    assert after < 0.8 * before
    assert all(p.grad is None for n, p in m.named_parameters() if "lora" not in n)


def test_online_learner_updates_adapters_while_decoding():
    m = _model(9, scale=0.0).float()
    learner = LowRankLearner(m, learning_rate=1e-2, interval=2)
    before = {n: p.clone() for n, p in m.named_parameters()}
    br = NoiseBranch(m, block_size=4)
    out = generate(br, torch.tensor([[5, 9, 13]]), 40, sampling=SamplingConfig(1.0),
                   generator=torch.Generator().manual_seed(1), feedback=LowRankFeedback(learner))
    assert len(out.tokens) == 40 and out.updates >= 1 and out.feedback_blocks >= 2
    changed = {n for n, p in m.named_parameters() if not torch.equal(before[n], p)}
    assert changed and all("lora" in n for n in changed)


def test_online_learner_loss_gradient_is_exact():
    m = _model(10).float()
    learner = LowRankLearner(m, interval=100)
    br = NoiseBranch(m, block_size=4)
    gen = torch.Generator().manual_seed(2)
    hist = m(torch.tensor([[4, 8, 15]])).cache
    d = br.draft(torch.tensor([[16]]), hist, 4, ProposalSampler(SamplingConfig(1.0)), gen,
                 feedback=LowRankFeedback(learner))
    teacher = m(d.verifier_inputs, cache=d.cache).logits[0]
    learner.observe(d.boundary, teacher, 3, may_update=False)
    assert learner.feedback_blocks == 1 and learner.updates == 0
    # recomputing the draft with the stored history reproduces the drafted rows
    again = m(d.boundary.inputs, cache=d.boundary.history, adapter_mask=d.boundary.route).logits
    direct = m(d.draft_inputs, cache=hist, adapter_mask=d.boundary.route).logits
    assert torch.allclose(again, direct)
    learner.step()
    assert learner.updates == 1 and learner.last_loss is not None


def test_checkpoint_roundtrip(tmp_path):
    m = _model(11).float()
    save(m, tmp_path / "m.pt")
    r = load(tmp_path / "m.pt")
    x = torch.tensor([[1, 2, 3]])
    assert torch.equal(r(x, adapter_mask=x > 1).logits, m(x, adapter_mask=x > 1).logits)
    torch.save({"format": "other"}, tmp_path / "bad.pt")
    with pytest.raises(ValueError):
        load(tmp_path / "bad.pt")


def test_hf_qwen3_backbone_imports_exactly():
    transformers = pytest.importorskip("transformers")
    cfg = transformers.Qwen3Config(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, head_dim=8,
                                   max_position_embeddings=128, tie_word_embeddings=False)
    torch.manual_seed(12)
    hf = transformers.Qwen3ForCausalLM(cfg).eval()
    m = from_hf(hf, dtype=torch.float32, adapter_rank=4)
    x = torch.tensor([[3, 9, 27, 17, 50, 2]])
    with torch.no_grad():
        want = hf(x).logits
    assert torch.allclose(m(x).logits, want, atol=1e-5)
    assert len(m.adapter_parameters()) == 2 * 7 * 2


def test_workspace_executor_matches_the_eager_branch():
    from online_speculation_b200.blockspec.lowrank_exec import GraphNoiseBranch

    m = _model(13)
    prompt = torch.tensor([[5, 9, 13, 2, 7, 1, 11, 4, 3, 8]])            # longer than a block: eager prefill
    eager = NoiseBranch(m, block_size=4)
    ws = GraphNoiseBranch(m, block_size=4, capacity=128)
    ws.prepare()
    for t in (0.0, 1.0):
        s = SamplingConfig(t)
        a = generate(eager, prompt, 25, sampling=s, generator=torch.Generator().manual_seed(3))
        b = generate(ws, prompt, 25, sampling=s, generator=torch.Generator().manual_seed(3))
        assert a.tokens == b.tokens and a.accepted_per_round == b.accepted_per_round
    assert ws.eager_forwards >= 1 and ws.graph_replays == 0
    assert generate_ar(ws, prompt, 12, sampling=SamplingConfig(0.0)).tokens == \
        generate_ar(eager, prompt, 12, sampling=SamplingConfig(0.0)).tokens
    with pytest.raises(ValueError):
        generate(ws, prompt, 200, sampling=SamplingConfig(0.0))              # past the capacity


def test_workspace_executor_learns_online_and_detects_storage_changes():
    from online_speculation_b200.blockspec.lowrank_exec import GraphNoiseBranch

    m = _model(14, scale=0.0).float()
    learner = LowRankLearner(m, learning_rate=1e-2, interval=2)
    ws = GraphNoiseBranch(m, block_size=4, capacity=128)
    out = generate(ws, torch.tensor([[5, 9, 13]]), 40, sampling=SamplingConfig(1.0),
                   generator=torch.Generator().manual_seed(1), feedback=LowRankFeedback(learner))
    assert out.updates >= 1 and any(float(p.abs().sum()) > 0 for n, p in m.named_parameters()
                                    if n.endswith("lora_B"))
    m.lm_head.weight.data = m.lm_head.weight.data.clone()
    with pytest.raises(RuntimeError):
        generate(ws, torch.tensor([[5, 9, 13]]), 4)


def test_peft_adapter_roundtrip(tmp_path):
    pytest.importorskip("safetensors")
    import json

    from online_speculation_b200.blockspec.lowrank import load_peft, save_peft

    m = _model(15).float()
    save_peft(m, tmp_path / "a")
    fresh = LowRankDecoder(m.config)
    fresh.load_state_dict({k: v for k, v in m.state_dict().items() if "lora" not in k}, strict=False)
    info = load_peft(fresh, tmp_path / "a")
    assert info["tensors"] == len(m.adapter_parameters())
    x = torch.tensor([[1, 2, 3, 4]])
    assert torch.equal(fresh(x, adapter_mask=x > 1).logits, m(x, adapter_mask=x > 1).logits)
    cfg = json.loads((tmp_path / "a" / "adapter_config.json").read_text())
    cfg["use_dora"] = True
    (tmp_path / "a" / "adapter_config.json").write_text(json.dumps(cfg))
    with pytest.raises(ValueError):
        load_peft(fresh, tmp_path / "a")
    other = LowRankDecoder(LowRankConfig(vocab_size=32, adapter_rank=4))
    cfg["use_dora"] = False
    (tmp_path / "a" / "adapter_config.json").write_text(json.dumps(cfg))
    with pytest.raises(ValueError):
        load_peft(other, tmp_path / "a")
