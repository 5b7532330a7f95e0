"""MoE layer and masked-diffusion model on the sm_100a kernels, against fp32 PyTorch."""
import math

import pytest
import torch

from online_speculation_b200.ops import kernels as ops

pytestmark = pytest.mark.gpu


def _grouped_case(E, M, K, counts, swiglu):
    torch.manual_seed(0)
    dev = "cuda"
    w = (torch.randn(E * M, K, device=dev) * 0.05).bfloat16()
    rows = sum(counts)
    x = torch.randn(rows, K, device=dev).bfloat16()
    offsets = torch.tensor([0] + list(torch.tensor(counts).cumsum(0).tolist()), dtype=torch.int32, device=dev)
    bn = ops.moe_pick_bn(rows, E)
    tiles = torch.zeros((M // 128) * (-(-rows // 32) + E) * 4, dtype=torch.int32, device=dev)
    total = torch.zeros(1, dtype=torch.int32, device=dev)
    ext = ops._ext.require()
    ext.grouped_tiles(offsets, E, M // 128, bn, tiles, total)
    out = torch.zeros(rows, M // 2 if swiglu else M, dtype=torch.bfloat16, device=dev)
    ws, ctr, st = ops.workspace.gemm_workspace(x.device), ops.workspace.gemm_counters(x.device), ops.workspace.status(
        x.device)
    ext.grouped_gemm(w, x, out, 1 if swiglu else 0, tiles, total, E, bn, ws, ctr, st)
    torch.cuda.synchronize()
    ref = torch.empty(rows, out.shape[1], device=dev)
    o = offsets.tolist()
    for e in range(E):
        if o[e + 1] > o[e]:
            ref[o[e]:o[e + 1]] = ops.linear_reference(x[o[e]:o[e + 1]], w[e * M:(e + 1) * M], swiglu=swiglu)
    return out.float(), ref


@pytest.mark.parametrize("swiglu", [False, True])
@pytest.mark.parametrize("counts", [[5, 0, 300, 64, 1, 0, 129, 40], [1000] * 4])
def test_grouped_gemm_matches_per_expert_fp32(swiglu, counts):
    got, ref = _grouped_case(len(counts), 256, 320, counts, swiglu)
    err = (got - ref).norm() / ref.norm()
    assert err < 0.01, float(err)


def test_moe_ffn_matches_reference():
    torch.manual_seed(1)
    dev = "cuda"
    T, H, F, E, k = 300, 256, 128, 8, 2
    x = torch.randn(T, H, device=dev).bfloat16()
    h = torch.randn(T, H, device=dev).bfloat16()
    router = (torch.randn(E, H, device=dev) * 0.5).bfloat16()
    gu = (torch.randn(E * 2 * F, H, device=dev) * 0.05).bfloat16()
    down = (torch.randn(E * H, F, device=dev) * 0.05).bfloat16()
    buf = ops.MoEBuffers(T, E, k, H, F, dev)
    got = ops.moe_ffn(x, h.clone(), router, gu, down, top_k=k, buffers=buf)
    # routing must agree with the fp32 reference where the k-th / (k+1)-th probabilities are separated
    idx_ref, w_ref = ops.moe_route_reference(x, router, k, False)
    idx = buf.idx[:T * k].view(T, k).long()
    probs = (x.float() @ router.float().t()).softmax(-1).sort(-1, descending=True).values
    clear = (probs[:, k - 1] - probs[:, k]) > 1e-3
    assert torch.equal(idx[clear], idx_ref[clear])
    ref = ops._moe_ffn_reference(x.cpu(), h.cpu().clone(), router.cpu(), gu.cpu(), down.cpu(), k, False)
    c = clear.cpu()
    d_got = got.float().cpu() - h.float().cpu()
    d_ref = ref.float() - h.float().cpu()
    err = (d_got - d_ref)[c].norm() / d_ref[c].norm()
    assert err < 0.02, float(err)
    # buffers are reusable: a second call gives the same result
    again = ops.moe_ffn(x, h.clone(), router, gu, down, top_k=k, buffers=buf)
    assert torch.equal(again, got)


def test_moe_diffusion_model_matches_fp32_reference():
    from online_speculation_b200.models.moe import PRESETS, MoEDiffusionModel, build_weights, random_state_dict, \
        reference_forward

    cfg = PRESETS["tiny-moe"]
    sd = random_state_dict(cfg, seed=2, std=0.05)
    model = MoEDiffusionModel(build_weights(cfg, sd, device="cuda"))
    toks = torch.randint(0, cfg.vocab_size, (2, 96), generator=torch.Generator().manual_seed(0))
    rows = torch.arange(32, 64).expand(2, 32)
    got = model.logits(toks.cuda(), rows.cuda()).cpu()
    for b in range(2):
        ref = reference_forward(cfg, sd, toks[b])[32:64]
        err = (got[b] - ref).norm() / ref.norm()
        assert err < 0.03, float(err)


def test_guided_logits_combine_hidden_rows():
    """CFG on the normalised hidden rows equals the logit-space combination u + (s+1)(c-u)."""
    from online_speculation_b200.models.moe import PRESETS, MoEDiffusionModel, build_weights, random_state_dict

    cfg = PRESETS["tiny-moe"]
    model = MoEDiffusionModel(build_weights(cfg, random_state_dict(cfg, seed=4), device="cuda"))
    torch.manual_seed(0)
    tok = torch.randint(0, cfg.vocab_size - 1, (3, 20), device="cuda")
    unc = tok.clone()
    unc[:, :6] = cfg.vocab_size - 1
    rows = torch.arange(8, 16, device="cuda").expand(3, 8)
    both = torch.cat((tok, unc))
    c, u = model.logits(both, torch.cat((rows, rows))).chunk(2)
    want = u + 2.5 * (c - u)
    got = model.logits(both, torch.cat((rows, rows)), guidance=1.5)
    assert got.shape == want.shape
    assert float((got - want).norm() / want.norm()) < 1e-2


def test_diffusion_backend_on_moe_engine():
    from online_speculation_b200.dllm import (DiffusionEngineBackend, DiffusionGenerationRequest,
                                              DiffusionSamplingConfig, DiffusionTrajectoryScoreRequest)
    from online_speculation_b200.models.moe import PRESETS, MoEDiffusionModel, build_weights, random_state_dict

    cfg = PRESETS["tiny-moe"]
    model = MoEDiffusionModel(build_weights(cfg, random_state_dict(cfg, seed=3), device="cuda"))
    be = DiffusionEngineBackend(model, model_id="tiny-moe")
    sp = DiffusionSamplingConfig(block_length=8, steps_per_block=4, temperature=1.0, remasking="random")
    reqs = [DiffusionGenerationRequest(tuple(range(5, 21)), 16, sp, seed=s, request_id=str(s)) for s in range(4)]
    out = be.sample_batch(reqs)
    scores = be.score_trajectories([DiffusionTrajectoryScoreRequest(s, sp) for s in out])
    for s, v in zip(out, scores):
        assert s.trajectory_logprob == pytest.approx(v, rel=1e-3, abs=1e-2)
        assert cfg.mask_token_id not in s.token_ids
    one = DiffusionEngineBackend(model, model_id="tiny-moe", max_batch_size=1).sample_batch(reqs)
    same = sum(a.token_ids == b.token_ids for a, b in zip(out, one))
    assert same >= 3   # batch-invariant draws (bf16 GEMM tiling may flip a near tie)
    greedy = DiffusionSamplingConfig(block_length=8, steps_per_block=8, temperature=0.0, cfg_scale=0.5)
    g = be.sample_batch([DiffusionGenerationRequest((3, 4, 5), 16, greedy, 0, "g")])[0]
    assert len(g.token_ids) == 16 and g.trajectory_logprob is None


def test_lora_linear_forward_backward_matches_fp32():
    from online_speculation_b200.training.lora import LoRAParameters, lora_linear

    torch.manual_seed(4)
    x = torch.randn(200, 256, device="cuda").bfloat16().requires_grad_(True)
    w = (torch.randn(384, 256, device="cuda") * 0.05).bfloat16()
    lo = LoRAParameters(256, 384, 8, groups=3, device="cuda")
    with torch.no_grad():
        lo.B.normal_(0, 0.1)
    y = lora_linear(x, w, lo, 2.0)
    gy = torch.randn_like(y)
    y.backward(gy)
    xf = x.detach().float().requires_grad_(True)
    A = lo.A.detach().clone().requires_grad_(True)
    B = lo.B.detach().clone().requires_grad_(True)
    yf = xf @ w.float().t() + 2.0 * (xf @ A.t()) @ (B * lo.block_mask).t()
    yf.backward(gy.float())
    assert (y.float() - yf).norm() / yf.norm() < 0.01
    for got, ref in ((x.grad.float(), xf.grad), (lo.A.grad, A.grad), (lo.B.grad, B.grad)):
        assert (got - ref).norm() / ref.norm() < 0.02


def test_lora_linear_dropout_keeps_the_base_gradient():
    """With adapter dropout the frozen product still passes its input gradient on."""
    from online_speculation_b200.training.lora import LoRAParameters, lora_linear

    torch.manual_seed(5)
    x = torch.randn(96, 256, device="cuda").bfloat16().requires_grad_(True)
    w = (torch.randn(128, 256, device="cuda") * 0.05).bfloat16()
    lo = LoRAParameters(256, 128, 8, device="cuda")
    with torch.no_grad():
        lo.B.normal_(0, 0.1)
    torch.manual_seed(11)
    y = lora_linear(x, w, lo, 2.0, dropout=0.3, training=True)
    gy = torch.randn_like(y)
    y.backward(gy)
    xf = x.detach().float().requires_grad_(True)
    A = lo.A.detach().clone().requires_grad_(True)
    B = lo.B.detach().clone().requires_grad_(True)
    torch.manual_seed(11)
    xa = torch.nn.functional.dropout(xf, 0.3, True)      # the same mask (same generator state, same call)
    yf = xf @ w.float().t() + 2.0 * (xa @ A.t()) @ (B * lo.block_mask).t()
    yf.backward(gy.float())
    assert (y.float() - yf).norm() / yf.norm() < 0.01
    for got, ref in ((x.grad.float(), xf.grad), (lo.A.grad, A.grad), (lo.B.grad, B.grad)):
        assert (got - ref).norm() / ref.norm() < 0.02


def test_vrpo_expert_adapters_on_gpu():
    """Expert gate / up / down adapters: GPU and CPU training steps agree."""
    from online_speculation_b200.dllm.config import VRPOSamplingConfig
    from online_speculation_b200.models.moe import PRESETS, build_weights, random_state_dict
    from online_speculation_b200.training.lora import LoRAConfig
    from online_speculation_b200.training.vrpo import VRPO_TARGETS, LoRAMoEPolicy, VRPOTrainer, VRPOTrainingConfig

    cfg = PRESETS["tiny-moe"]
    sd = random_state_dict(cfg, seed=7)
    lora = LoRAConfig(rank=8, targets=VRPO_TARGETS)
    gpu = LoRAMoEPolicy(build_weights(cfg, sd, device="cuda"), lora)
    cpu = LoRAMoEPolicy(build_weights(cfg, sd, device="cpu"), lora)
    g = torch.Generator().manual_seed(2)
    pairs = [tuple(tuple(torch.randint(0, 500, (n,), generator=g).tolist()) for n in (32, 32, 32))]
    conf = VRPOTrainingConfig(learning_rate=1e-3, gradient_accumulation_steps=1,
                              sampling=VRPOSamplingConfig(timestep_samples=4))
    tg, tc = VRPOTrainer(gpu, pairs, conf), VRPOTrainer(cpu, pairs, conf)
    rg, rc = tg.train_step(), tc.train_step()
    assert rg["loss"] == pytest.approx(math.log(2), abs=1e-4)
    assert rg["grad_norm"] == pytest.approx(rc["grad_norm"], rel=0.1)
    r2 = tg.train_step()
    assert math.isfinite(r2["loss"]) and r2["preference_score"] != 0.0


def test_moe_autograd_backward_matches_reference():
    from online_speculation_b200.training.moe_autograd import FrozenExperts, _moe_reference_autograd, \
        moe_ffn_autograd

    torch.manual_seed(5)
    T, H, Fd, E, k = 160, 256, 128, 8, 2
    router = (torch.randn(E, H) * 0.5).bfloat16()
    gu = (torch.randn(E * 2 * Fd, H) * 0.05).bfloat16()
    down = (torch.randn(E * H, Fd) * 0.05).bfloat16()
    x0 = torch.randn(T, H).bfloat16()
    h0 = torch.randn(T, H).bfloat16()
    gout = torch.randn(T, H)
    exg = FrozenExperts(router.cuda(), gu.cuda(), down.cuda(), k, False)
    x = x0.cuda().requires_grad_(True)
    h = h0.cuda().requires_grad_(True)
    out = moe_ffn_autograd(x, h, exg, torch.zeros((), device="cuda", requires_grad=True))
    out.float().backward(gout.cuda())
    exc = FrozenExperts(router, gu, down, k, False)
    xc = x0.float().requires_grad_(True)
    hc = h0.float().requires_grad_(True)
    outc = _moe_reference_autograd(xc, hc, exc)
    outc.float().backward(gout)
    assert (out.float().cpu() - outc.float()).norm() / outc.float().norm() < 0.02
    assert (x.grad.float().cpu() - xc.grad).norm() / xc.grad.norm() < 0.05
    assert torch.allclose(h.grad.float().cpu(), hc.grad, atol=1e-2)


def test_vrpo_step_on_gpu():
    from online_speculation_b200.dllm.config import VRPOSamplingConfig
    from online_speculation_b200.models.moe import PRESETS, build_weights, random_state_dict
    from online_speculation_b200.training.lora import LoRAConfig
    from online_speculation_b200.training.vrpo import LoRAMoEPolicy, VRPOTrainer, VRPOTrainingConfig

    cfg = PRESETS["tiny-moe"]
    sd = random_state_dict(cfg, seed=6)
    gpu = LoRAMoEPolicy(build_weights(cfg, sd, device="cuda"), LoRAConfig(rank=8))
    cpu = LoRAMoEPolicy(build_weights(cfg, sd, device="cpu"), LoRAConfig(rank=8))
    g = torch.Generator().manual_seed(1)
    pairs = [tuple(tuple(torch.randint(0, 500, (n,), generator=g).tolist()) for n in (32, 32, 32))]
    conf = VRPOTrainingConfig(learning_rate=1e-3, gradient_accumulation_steps=1,
                              sampling=VRPOSamplingConfig(timestep_samples=4))
    tg, tc = VRPOTrainer(gpu, pairs, conf), VRPOTrainer(cpu, pairs, conf)
    rg, rc = tg.train_step(), tc.train_step()
    assert rg["loss"] == pytest.approx(math.log(2), abs=1e-4)
    assert rg["grad_norm"] == pytest.approx(rc["grad_norm"], rel=0.1)
    r2 = tg.train_step()
    assert math.isfinite(r2["loss"]) and r2["preference_score"] != 0.0
