"""The batched runner and the speculative MH engine against the fp32 oracle."""

import math

import pytest
import torch

from online_speculation_b200.api import build_mh_engine
from online_speculation_b200.engine.kv_cache import KVCache
from online_speculation_b200.engine.runner import ModelRunner, build_meta
from online_speculation_b200.models.decoder import PRESETS, DecoderConfig, build_weights, random_state_dict, reference_forward
from online_speculation_b200.ops import workspace

pytestmark = pytest.mark.gpu

SMALL = DecoderConfig(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=3,
                      num_attention_heads=8, num_key_value_heads=2, name="small")
SMALL_QK = DecoderConfig(vocab_size=1024, hidden_size=512, intermediate_size=768, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=4, attention_bias=False, qk_norm=True,
                         tie_word_embeddings=True, name="small-qk")


def _setup(cfg, seed=0):
    sd = random_state_dict(cfg, seed=seed, std=0.05, device="cpu")
    w = build_weights(cfg, sd, device="cuda")
    cache = KVCache(cfg.num_hidden_layers, w.heads.kv_slots, 64, "cuda")
    return sd, ModelRunner(w, cache, max_tokens=1024)


@pytest.mark.parametrize("cfg", [SMALL, SMALL_QK])
def test_prefill_decode_verify_match_oracle(cfg):
    sd, r = _setup(cfg)
    torch.manual_seed(0)
    seq = torch.randint(0, cfg.vocab_size, (70,))
    ref = reference_forward(cfg, sd, seq)                       # [70, V] fp32
    G = r.q_slots // r.kv_slots
    cache = r.cache
    s = cache.create()
    # prefill 60 tokens (logits for all rows)
    slots = cache.append(s, 60)
    table = torch.zeros(1, 8, dtype=torch.int32)
    cache.fill_table([s], table)
    meta = build_meta("cuda", table, seq[:60].tolist(), list(range(60)), slots, [60], [60], [0], G)
    out = r.forward(meta)
    rel = float((out.cpu() - ref[:60]).norm() / ref[:60].norm())
    assert rel < 3e-2
    # one decode step
    slots = cache.append(s, 1)
    cache.fill_table([s], table)
    meta = build_meta("cuda", table, [int(seq[60])], [60], slots, [1], [61], [0], G)
    out = r.forward(meta)
    assert float((out.cpu()[0] - ref[60]).norm() / ref[60].norm()) < 3e-2
    # a causal verify block of 4
    slots = cache.append(s, 4)
    cache.fill_table([s], table)
    meta = build_meta("cuda", table, seq[61:65].tolist(), list(range(61, 65)), slots, [4], [65], [0], G)
    out = r.forward(meta)
    assert float((out.cpu() - ref[61:65]).norm() / ref[61:65].norm()) < 3e-2
    torch.cuda.synchronize()
    workspace.check_status()


def test_forked_sequences_share_prefix_pages():
    sd, r = _setup(SMALL)
    cache = r.cache
    G = r.q_slots // r.kv_slots
    torch.manual_seed(1)
    seq = torch.randint(0, SMALL.vocab_size, (80,))
    ref = reference_forward(SMALL, sd, seq)
    s = cache.create()
    slots = cache.append(s, 45)
    table = torch.zeros(1, 8, dtype=torch.int32)
    cache.fill_table([s], table)
    r.forward(build_meta("cuda", table, seq[:45].tolist(), list(range(45)), slots, [45], [45], [0], G),
              compute_logits=False)
    f = cache.fork(s, 40)          # shares page 0, copies 8 tokens of page 1
    assert cache.manager.refcount(cache.manager.pages(s)[0]) == 2
    cache.flush_copies()
    slots = cache.append(f, 1)
    cache.fill_table([f], table)
    out = r.forward(build_meta("cuda", table, [int(seq[40])], [40], slots, [1], [41], [0], G))
    assert float((out.cpu()[0] - ref[40]).norm() / ref[40].norm()) < 3e-2
    cache.release(s)
    cache.release(f)
    assert cache.free_pages == cache.num_pages


@pytest.mark.parametrize("graphs,policy", [(False, "always"), (True, "always"), (True, "adaptive")])
def test_mh_engine_logprobs_are_exact(graphs, policy):
    """Every emitted token's log p / log q must equal the oracle's log-softmax of the chain prefix."""
    cfg = SMALL
    eng = build_mh_engine(cfg, seed=3, alpha=2.0, length=24, block_size=4, learner_stride=8, use_graphs=graphs,
                          kv_bytes=64 << 20, max_seq_tokens=64, max_batch=8, spec_policy=policy, probe_every=3)
    prompt = list(range(5, 21))
    eng.add_chains([prompt] * 6)
    eng.run_until_idle()
    eng.set_quota(3)
    eng.run_until_idle()
    assert eng.stats["mh_updates"] == 18
    assert eng.learner.updates >= 1
    # the oracle uses the same random weights (drawn on the same device from the same seed)
    sd = {k: v.cpu() for k, v in random_state_dict(cfg, seed=3, std=0.02, device="cuda").items()}
    for ch in eng.chains:
        assert len(ch.tokens) == 24
        full = torch.tensor(ch.prompt + ch.tokens)
        logits = reference_forward(cfg, sd, full)[len(prompt) - 1:-1]
        lp = logits.log_softmax(-1).gather(-1, torch.tensor(ch.tokens)[:, None]).squeeze(-1)
        lq = (logits * 2.0).log_softmax(-1).gather(-1, torch.tensor(ch.tokens)[:, None]).squeeze(-1)
        assert torch.allclose(torch.tensor(ch.logp), lp, atol=0.05)
        assert torch.allclose(torch.tensor(ch.logq), lq, atol=0.1)
    # pages: each chain holds its state, nothing leaked
    held = sum(1 for p in range(eng.cache.num_pages) if eng.cache.manager.refcount(p) > 0)
    assert held <= 6 * 2 + 2
    assert eng.mean_accept_length >= 1.0
    if policy == "adaptive":
        assert eng.stats["spec_rounds"] > 0 and eng.stats["plain_rounds"] > 0
    workspace.check_status()


@pytest.mark.parametrize("policy", ["always", "never"])
def test_mh_engine_shared_prompt_two_pass_attention_is_exact(policy):
    """A 160-token prompt shared by every chain: attention reads its 128 full-page keys in one shared
    pass; the emitted tokens' log p / log q still equal the oracle's."""
    cfg = SMALL
    eng = build_mh_engine(cfg, seed=3, alpha=2.0, length=20, block_size=4, learner_stride=None, use_graphs=True,
                          kv_bytes=64 << 20, max_seq_tokens=200, max_batch=8, spec_policy=policy, share_prefix=True)
    prompt = [(7 * i) % 900 + 5 for i in range(160)]
    eng.add_chains([prompt] * 5)
    assert eng.shared_prefix_keys == 128
    eng.run_until_idle()
    eng.set_quota(2)
    eng.run_until_idle()
    sd = {k: v.cpu() for k, v in random_state_dict(cfg, seed=3, std=0.02, device="cuda").items()}
    for ch in eng.chains:
        full = torch.tensor(ch.prompt + ch.tokens)
        logits = reference_forward(cfg, sd, full)[len(prompt) - 1:-1]
        lp = logits.log_softmax(-1).gather(-1, torch.tensor(ch.tokens)[:, None]).squeeze(-1)
        # bf16 activations over a 180-token context against the fp32 oracle
        assert torch.allclose(torch.tensor(ch.logp), lp, atol=0.1)
    eng.close()
    workspace.check_status()


def test_mh_engine_without_draft_is_exact():
    """Plain decoding (no draft head) emits one token per round with exact log p / log q."""
    cfg = SMALL
    eng = build_mh_engine(cfg, seed=3, alpha=2.0, length=16, use_graphs=True, kv_bytes=64 << 20, max_seq_tokens=64,
                          max_batch=8, draft=False)
    prompt = list(range(5, 21))
    eng.add_chains([prompt] * 4)
    eng.run_until_idle()
    eng.set_quota(2)
    eng.run_until_idle()
    assert eng.stats["mh_updates"] == 8 and eng.stats["spec_rounds"] == 0 and eng.stats["plain_rounds"] > 0
    sd = {k: v.cpu() for k, v in random_state_dict(cfg, seed=3, std=0.02, device="cuda").items()}
    for ch in eng.chains:
        full = torch.tensor(ch.prompt + ch.tokens)
        logits = reference_forward(cfg, sd, full)[len(prompt) - 1:-1]
        lp = logits.log_softmax(-1).gather(-1, torch.tensor(ch.tokens)[:, None]).squeeze(-1)
        lq = (logits * 2.0).log_softmax(-1).gather(-1, torch.tensor(ch.tokens)[:, None]).squeeze(-1)
        assert torch.allclose(torch.tensor(ch.logp), lp, atol=0.05)
        assert torch.allclose(torch.tensor(ch.logq), lq, atol=0.1)
    eng.close()
    workspace.check_status()


def test_online_learner_raises_acceptance():
    """A draft copied from the target's last attention and then corrupted with noise recovers
    acceptance through the online learner."""
    from online_speculation_b200.api import build_runner
    from online_speculation_b200.engine.draft import DraftHead, SuffixConfig, SuffixLearner, init_draft
    from online_speculation_b200.engine.mh_engine import MHEngine

    cfg = SMALL
    runner = build_runner(cfg, seed=4, kv_bytes=128 << 20, max_tokens=2048)
    draft = init_draft(runner.w, seed=5, copy_from_target=True)
    g = torch.Generator(device="cuda").manual_seed(6)
    for name in ("w_qkv", "w_o"):
        t = getattr(draft, name)
        noise = torch.randn(t.shape, generator=g, device="cuda") * float(t.float().std())
        t.copy_((t.float() + noise * (t != 0).float()).to(t.dtype))
    head = DraftHead(runner, draft, block_size=4)
    learner = SuffixLearner(head, SuffixConfig(stride=4, learning_rate=2e-3), use_graphs=True)
    eng = MHEngine(runner, head, alpha=4.0, length=64, root_seed=7, learner=learner, use_graphs=True,
                   max_pages_per_seq=8, spec_policy="always")
    eng.add_chains([list(range(5, 37))] * 8)
    eng.set_quota(10_000)

    def window(rounds):
        b0, e0 = eng.stats["blocks"], eng.stats["emitted"]
        for _ in range(rounds):
            eng.round()
        return (eng.stats["emitted"] - e0) / max(1, eng.stats["blocks"] - b0)

    before = window(50)
    window(500)
    after = window(50)
    print(f"accept length before {before:.3f} after {after:.3f}, learner updates {learner.updates}")
    assert learner.updates >= 100
    assert after > before + 0.05
    eng.close()
    workspace.check_status()


def test_kernel_branch_matches_module_branch():
    from online_speculation_b200.blockspec.generation import MaskedAttentionBranch, ProposalSampler, generate
    from online_speculation_b200.blockspec.kernel_branch import KernelBranch
    from online_speculation_b200.blockspec.model import DualViewConfig, DualViewDecoder
    from online_speculation_b200.blockspec.sampling import SamplingConfig

    cfg = DualViewConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=128, block_size=4, mask_token_id=1)
    torch.manual_seed(0)
    m = DualViewDecoder(cfg).cuda().eval().requires_grad_(False)
    with torch.no_grad():
        for layer in m.layers:
            layer.attention.draft.q.weight.mul_(1.3)
    mb, kb = MaskedAttentionBranch(m), KernelBranch(m, kv_bytes=64 << 20)
    prompt = torch.tensor([[3, 7, 11, 13, 17]], device="cuda")
    l1, c1 = mb.ar(prompt)
    l2, c2 = kb.ar(prompt)
    assert float((l1 - l2).norm() / l1.norm()) < 3e-2
    anchor = torch.tensor([[19]], device="cuda")
    sampler = ProposalSampler(SamplingConfig(0.0))
    d1 = mb.draft(anchor, c1, 4, sampler)
    d2 = kb.draft(anchor, c2, 4, sampler)
    assert kb.cache_length(c2) == 5
    out1 = m(d1.verifier_inputs, cache=c1)
    l3, _ = kb.ar(d1.verifier_inputs, cache=c2)
    assert float((out1.logits - l3).norm() / out1.logits.norm()) < 3e-2
    # full speculative generation runs on the kernel branch
    res = generate(kb, prompt, 16, sampling=SamplingConfig(1.0), generator=torch.Generator(device="cuda").manual_seed(0))
    assert len(res.tokens) == 16


def test_learner_draft_attention_matches_fp32():
    from online_speculation_b200.engine.draft import FeedbackRound, SuffixLearner

    torch.manual_seed(0)
    dev = torch.device("cuda")
    B, Kb, qs, ks, D, P = 5, 4, 8, 2, 128, 3
    pages = B * P + 2
    kc = torch.randn(pages, ks, 32, D, device=dev).bfloat16()
    vc = torch.randn(pages, ks, 32, D, device=dev).bfloat16()
    table = torch.randperm(pages, device=dev)[:B * P].view(B, P).int()
    hist = torch.tensor([0, 5, 32, 70, 95], device=dev)
    positions = (hist[:, None] + torch.arange(Kb, device=dev)[None]).int()
    q = torch.randn(B, Kb, qs, D, device=dev, requires_grad=True)
    k = torch.randn(B, Kb, ks, D, device=dev, requires_grad=True)
    v = torch.randn(B, Kb, ks, D, device=dev, requires_grad=True)
    fb = FeedbackRound(None, positions, table, None, None, None, B)
    out = SuffixLearner._draft_attention(q, k, v, fb, kc, vc).float()
    # fp32 oracle
    ref = torch.zeros(B, Kb, qs, D, device=dev)
    for b in range(B):
        n = int(hist[b])
        hk = kc[table[b].long()].permute(1, 0, 2, 3).reshape(ks, P * 32, D)[:, :n].float()
        hv = vc[table[b].long()].permute(1, 0, 2, 3).reshape(ks, P * 32, D)[:, :n].float()
        keys = torch.cat((hk, k[b].permute(1, 0, 2)), 1)
        vals = torch.cat((hv, v[b].permute(1, 0, 2)), 1)
        for h in range(qs):
            g = h // (qs // ks)
            s = (q[b, :, h] @ keys[g].T) * D ** -0.5
            ref[b, :, h] = s.softmax(-1) @ vals[g]
    ref = ref.reshape(B, Kb, qs * D)
    assert float((out - ref).norm() / ref.norm()) < 2e-2
    # gradients flow to the block's q, k and v
    (out * torch.randn_like(out)).sum().backward()
    assert q.grad is not None and k.grad.abs().sum() > 0 and v.grad.abs().sum() > 0
