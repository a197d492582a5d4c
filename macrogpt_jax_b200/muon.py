"""Muon's orthogonalisation (ueaj/opt/multiscale.py:110-200) on this package's kernels.

Same names and arguments as the reference:
  orthogonalize(x, ns_steps=5, eps=1e-8, method='muon' | 'optimal', convergence_speed=1e-3)
      multiscale.py:110-141: optax 0.2.6's orthogonalize_via_newton_schulz mapped over the leading
      axes of x (a 2-D x is one slice; more than 3 dimensions are flattened to [-1, m, n]);
      'muon' uses the fixed coefficients (3.4445, -4.7750, 2.0315) for every step, 'optimal' the
      per-step coefficients of optimal_composition(convergence_speed, ns_steps).
  optimal_quintic(l, u), optimal_composition(min_orth, num_iters, cushion)   multiscale.py:144-200
      the host-side computation of those coefficients (float64 here; the reference evaluates them
      with jnp, float32 by default, so they agree to ~1e-7 relative).

The iteration itself is ufp8_newton_schulz (csrc/ns.cu): three bf16 tcgen05 GEMMs per step with
the updates in their epilogues, batched over the slices, x's dtype (f32 or bf16) in and out.
"""
from __future__ import annotations

from functools import lru_cache
from typing import Literal, Optional

import numpy as np
import torch

from . import ops

MUON_COEFFS = (3.4445, -4.7750, 2.0315)


def optimal_quintic(l: float, u: float):
    """Coefficients (a, b, c) of the odd quintic a x + b x^3 + c x^5 that maps [l, u] closest to 1
    in the equioscillation sense (multiscale.py:144-175): alternate between solving the 4 x 4
    system for (a, b, c, E) at the nodes l, q, r, u and moving q, r to the polynomial's extrema,
    until E stops changing."""
    if not 0 <= l <= u:
        raise ValueError(f"optimal_quintic needs 0 <= l <= u, got {l}, {u}")
    if 1 - 5e-6 <= l / u:
        return (15 / 8) / u, (-10 / 8) / (u ** 3), (3 / 8) / (u ** 5)
    q, r = (3 * l + 1) / 4, (l + 3) / 4
    E, old_E = np.inf, None
    count = 0
    while not old_E or abs(old_E - E) > 1e-15:
        old_E = E
        lhs = np.array([[l, l ** 3, l ** 5, 1.0],
                        [q, q ** 3, q ** 5, -1.0],
                        [r, r ** 3, r ** 5, 1.0],
                        [u, u ** 3, u ** 5, -1.0]], dtype=np.float64)
        a, b, c, E = np.linalg.solve(lhs, np.ones(4))
        disc = np.sqrt(9 * b ** 2 - 20 * a * c)
        q, r = np.sqrt((-3 * b + np.array([-1.0, 1.0]) * disc) / (10 * c))
        count += 1
        if count > 1000:
            raise ValueError(f"Failed to converge after {count} iterations.")
    return float(a), float(b), float(c)


@lru_cache
def optimal_composition(min_orth: float, num_iters: int, cushion: float = 0.02407327424182761):
    """Per-step coefficients (multiscale.py:178-200): each step's quintic is optimal on
    [max(min_orth, cushion u), u], rescaled so that it is centred on 1 over [min_orth, u]; then
    min_orth and u move to that polynomial's image."""
    u = 1.0
    coefficients = []
    for _ in range(num_iters):
        a, b, c = optimal_quintic(max(min_orth, cushion * u), u)
        pl = a * min_orth + b * min_orth ** 3 + c * min_orth ** 5
        pu = a * u + b * u ** 3 + c * u ** 5
        rescalar = 2 / (pl + pu)
        a, b, c = a * rescalar, b * rescalar, c * rescalar
        coefficients.append((a, b, c))
        min_orth = a * min_orth + b * min_orth ** 3 + c * min_orth ** 5
        u = 2 - min_orth
    return tuple(coefficients)


def ns_coefficients(ns_steps: int = 5, method: Literal["muon", "optimal"] = "muon",
                    convergence_speed: Optional[float] = 1e-3):
    if method == "muon":
        return (MUON_COEFFS,) * ns_steps
    if method == "optimal":
        return optimal_composition(convergence_speed, ns_steps)
    raise ValueError(f"Unknown value for `method`: {method}")


def orthogonalize(x: torch.Tensor, ns_steps: int = 5, eps: float = 1e-8,
                  method: Literal["muon", "optimal"] = "muon",
                  convergence_speed: Optional[float] = 1e-3) -> torch.Tensor:
    """Newton-Schulz orthogonalisation of every [m, n] slice of x (multiscale.py:110-141); x is a
    CUDA f32 or bf16 tensor with ndim >= 2, the result has its shape and dtype."""
    coeffs = ns_coefficients(ns_steps, method, convergence_speed)
    shape = x.shape
    if x.dim() <= 1:
        raise ValueError(f"Input must have shape (m, n), got {tuple(shape)}")
    x3 = x.reshape((-1,) + tuple(shape[-2:]))
    return ops.newton_schulz(x3, coeffs, eps).reshape(shape)
