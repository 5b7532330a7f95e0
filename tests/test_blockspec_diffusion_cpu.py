"""Discrete corruption kernels (CPU): the reverse posterior against brute-force Bayes over the
forward chain, the predictor-corrector blend, corruption rates and noise bounds."""

import pytest
import torch

from online_speculation_b200.blockspec.diffusion import UniformNoise, corrupt, posterior, psi_transition


def _chain(x, prior, alpha):
    """q(z | x) of the reset-to-prior forward process as a vector."""
    v = (1 - alpha) * prior.clone()
    v[x] += alpha
    return v


def test_posterior_is_bayes_over_the_forward_chain():
    g = torch.Generator().manual_seed(0)
    V = 5
    prior = torch.softmax(torch.randn(V, generator=g, dtype=torch.float64), -1)
    a_s, a_t = 0.7, 0.3
    r = a_t / a_s
    for x in range(V):
        qs = _chain(x, prior, a_s)                       # q(z_s | x)
        step = r * torch.eye(V, dtype=torch.float64) + (1 - r) * prior[None, :]   # q(z_t | z_s) rows
        joint = qs[:, None] * step                       # [z_s, z_t]
        for zt in range(V):
            want = joint[:, zt] / joint[:, zt].sum()
            got = posterior(torch.tensor(zt), torch.nn.functional.one_hot(torch.tensor(x), V).double(), prior,
                            a_s, a_t)
            assert torch.allclose(got, want, atol=1e-12)
        # the two steps compose to the direct corruption to alpha_t
        assert torch.allclose(qs @ step, _chain(x, prior, a_t), atol=1e-12)


def test_psi_transition_blends_ancestral_and_corrector():
    g = torch.Generator().manual_seed(1)
    V = 6
    prior = torch.full((V,), 1.0 / V, dtype=torch.float64)
    clean = torch.softmax(torch.randn(3, V, generator=g, dtype=torch.float64), -1)
    zt = torch.tensor([0, 3, 5])
    anc = posterior(zt, clean, prior, 0.8, 0.4)
    assert torch.allclose(psi_transition(zt, clean, prior, 0.8, 0.4, kappa=1.0), anc)
    mid = psi_transition(zt, clean, prior, 0.8, 0.4, kappa=0.5)
    assert torch.allclose(mid.sum(-1), torch.ones(3, dtype=torch.float64)) and bool((mid >= 0).all())
    corr = 0.8 * posterior(zt, clean, prior, 1.0, 0.4) + 0.2 * prior
    assert torch.allclose(psi_transition(zt, clean, prior, 0.8, 0.4, kappa=0.0), corr)
    with pytest.raises(ValueError):
        posterior(zt, clean, prior, 0.4, 0.8)


def test_corruption_rate_and_noise_bounds():
    g = torch.Generator().manual_seed(2)
    clean = torch.zeros(20000, dtype=torch.long)
    prior = torch.tensor([0.0, 0.5, 0.5])
    z = corrupt(clean, prior, 0.3, generator=g)
    assert float((z == 0).float().mean()) == pytest.approx(0.3, abs=0.02)   # only survivors keep token 0
    n = UniformNoise(2, 5).sample((1000,), 10, device="cpu", generator=g)
    assert int(n.min()) >= 2 and int(n.max()) <= 4
    with pytest.raises(ValueError):
        UniformNoise(3, 3)
    with pytest.raises(ValueError):
        UniformNoise(0, 20).sample((2,), 10, device="cpu")
