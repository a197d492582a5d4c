"""Muon's Newton-Schulz orthogonalisation restated on the CPU (oracle; test infrastructure only).

Follows ueaj/opt/multiscale.py:110-141, which maps optax 0.2.6's
contrib orthogonalize_via_newton_schulz (requirements.txt:45; its published algorithm: transpose a
tall slice, divide by its Frobenius norm + eps, then per step A = X X^T, B = b A + c A A,
X = a X + B X, transpose back) over the leading axes, with the coefficient sets of
multiscale.py:118-124 ('muon': the fixed triple; 'optimal': optimal_composition, restated below
from multiscale.py:144-200 in float64).

Two evaluations:
  * orthogonalize_f64: the algorithm in float64 (the reference's own arithmetic is f32 with XLA's
    matmul precision; neither JAX nor optax runs here, so parity with it is unpinned);
  * orthogonalize_bf16: the kernel's storage points, so the GPU can be held to a tight bar: X, A
    and B rounded to bf16 after each product, products accumulated in float64, the epilogue's
    f32 operations (alpha * acc + beta * C, each product and the sum rounded once), and the
    normalisation x / (sqrt(sum x^2) + eps) in f32 before the bf16 rounding.
"""
from __future__ import annotations

import numpy as np

from .fp8 import round_bf16

MUON = (3.4445, -4.7750, 2.0315)


def optimal_quintic(l, u):
    assert 0 <= l <= u
    if 1 - 5e-6 <= l / u:
        return (15 / 8) / u, (-10 / 8) / (u ** 3), (3 / 8) / (u ** 5)
    q, r = (3 * l + 1) / 4, (l + 3) / 4
    E, old_E = np.inf, None
    it = 0
    while not old_E or abs(old_E - E) > 1e-15:
        old_E = E
        m = np.array([[l, l ** 3, l ** 5, 1.0], [q, q ** 3, q ** 5, -1.0],
                      [r, r ** 3, r ** 5, 1.0], [u, u ** 3, u ** 5, -1.0]])
        a, b, c, E = np.linalg.solve(m, np.ones(4))
        q, r = np.sqrt((-3 * b + np.array([-1.0, 1.0]) * np.sqrt(9 * b ** 2 - 20 * a * c)) / (10 * c))
        it += 1
        assert it <= 1000
    return float(a), float(b), float(c)


def optimal_composition(min_orth, num_iters, cushion=0.02407327424182761):
    u, out = 1.0, []
    for _ in range(num_iters):
        a, b, c = optimal_quintic(max(min_orth, cushion * u), u)
        k = 2 / ((a * min_orth + b * min_orth ** 3 + c * min_orth ** 5) + (a * u + b * u ** 3 + c * u ** 5))
        a, b, c = a * k, b * k, c * k
        out.append((a, b, c))
        min_orth = a * min_orth + b * min_orth ** 3 + c * min_orth ** 5
        u = 2 - min_orth
    return out


def coefficients(steps=5, method="muon", convergence_speed=1e-3):
    return [MUON] * steps if method == "muon" else optimal_composition(convergence_speed, steps)


def orthogonalize_f64(g: np.ndarray, coeffs, eps=1e-8, dtype=np.float64) -> np.ndarray:
    """[batch, m, n] -> [batch, m, n], evaluated in `dtype` (float64 for parity checks, float32
    for the timed CPU baseline)."""
    out = np.empty(g.shape, dtype)
    for i, x in enumerate(np.asarray(g, dtype)):
        tr = x.shape[0] > x.shape[1]
        if tr:
            x = x.T
        x = (x / (np.linalg.norm(x) + dtype(eps))).astype(dtype)
        for a, b, c in coeffs:
            A = x @ x.T
            B = b * A + c * (A @ A)
            x = a * x + B @ x
        out[i] = x.T if tr else x
    return out


def _axpby(acc, alpha, beta, cm):
    """The AXPBY epilogue in f32: alpha * acc + beta * C, each product and the sum rounded once."""
    f = np.float32
    return (acc.astype(f) * f(alpha)).astype(f) + (cm.astype(f) * f(beta)).astype(f)


def orthogonalize_bf16(g: np.ndarray, coeffs, eps=1e-8, out_f32=True) -> np.ndarray:
    """The kernel's storage points (see the module docstring); returns f32 values."""
    f = np.float32
    out = np.empty(g.shape, f)
    for i, x in enumerate(np.asarray(g, f)):
        tr = x.shape[0] > x.shape[1]
        # normalisation on the stored layout: per-element f32 division by sqrt(sum) + eps
        ss = f((x.astype(np.float64) ** 2).sum())
        dn = f(f(np.sqrt(ss)) + f(eps))
        X = round_bf16((x / dn).astype(f))
        for k, (a, b, c) in enumerate(coeffs):
            Xs = X.T if tr else X
            A = round_bf16((Xs.astype(np.float64) @ Xs.T.astype(np.float64)).astype(f))
            A64 = A.astype(np.float64)
            B = round_bf16(_axpby(A64 @ A64.T, c, b, A))
            if tr:
                acc = X.astype(np.float64) @ B.astype(np.float64)  # X B (B symmetric)
            else:
                acc = B.astype(np.float64) @ X.astype(np.float64)
            Xn = _axpby(acc, 1.0, a, X)
            last = k == len(coeffs) - 1
            X = Xn if (last and out_f32) else round_bf16(Xn)
        out[i] = X
    return out
