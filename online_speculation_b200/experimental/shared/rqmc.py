"""Randomized quasi-Monte Carlo uniforms for rollout designs.

* ``randomized_lattice_uniforms(n, seed)``: one uniform shift s and the points
  (s + i / n) mod 1; each point is marginally U[0, 1) and the n points are
  evenly spaced on the circle.  An arithmetic-coding sampler maps each point to
  a full sequence.
* ``scrambled_sobol_uniforms(n, d, seed)``: an Owen-scrambled Sobol net in
  [0, 1)^d, one coordinate per generated token (inverse-CDF sampling).

Reference behaviour: src/inference_scaling/experimental/shared/rqmc.py:8-52.
"""

from __future__ import annotations

import numpy as np
import torch

_BELOW_ONE = float(np.nextafter(1.0, 0.0))


def randomized_lattice_uniforms(count: int, *, seed: int) -> tuple[float, ...]:
    if count <= 0:
        raise ValueError("lattice count must be positive")
    if seed < 0:
        raise ValueError("lattice seed must be non-negative")
    shift = float(np.random.default_rng(seed).random())
    pts = np.mod(shift + np.arange(count, dtype=np.float64) / count, 1.0)
    return tuple(float(min(p, _BELOW_ONE)) for p in pts)


def scrambled_sobol_uniforms(count: int, dimension: int, *, seed: int) -> tuple[tuple[float, ...], ...]:
    if count <= 0 or dimension <= 0:
        raise ValueError("Sobol count and dimension must be positive")
    if seed < 0:
        raise ValueError("Sobol seed must be non-negative")
    eng = torch.quasirandom.SobolEngine(dimension=dimension, scramble=True, seed=int(seed % (2 ** 31 - 1)))
    pts = np.minimum(eng.draw(count, dtype=torch.float64).numpy(), _BELOW_ONE)
    return tuple(tuple(float(v) for v in row) for row in pts)


__all__ = ["randomized_lattice_uniforms", "scrambled_sobol_uniforms"]
