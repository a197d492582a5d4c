"""RMSNorm restated on the CPU (oracle; test infrastructure only).

Follows RMSNorm.__call__ (ueaj/model/rmsnorm.py:68-84): x in f32, var = mean(x^2),
x * rsqrt(var + eps), times scale (uncentered) or 1 + scale (centered, rmsnorm.py:80-83), cast
back to the input dtype (bf16).  Where the reference leaves the arithmetic unspecified (XLA
chooses the reduction order of jnp.mean and the rsqrt implementation), this restatement fixes
it, and the CUDA kernel (csrc/norm.cu) follows the same choices bit for bit:
  * the sum of squares of a row: lane l of 32 accumulates, in increasing index order, the
    elements of the 8-element chunks c with c % 32 == l (f32, each product and sum rounded on
    its own), then the 32 lane sums are combined by an xor butterfly over offsets 16, 8, 4, 2, 1;
  * rsqrt(v) = 1 / sqrt(v) with an IEEE square root and IEEE divisions (var = ss / d).
Parity against the reference's own JAX output is unpinned (JAX cannot run here).
"""
from __future__ import annotations

import numpy as np

from .fp8 import bf16_bits_to_f32, f32_to_bf16_bits, quantize_bits


def _weight(scale_bits, centered: bool, d: int) -> np.ndarray:
    if scale_bits is None:
        return np.ones(d, np.float32)
    s = bf16_bits_to_f32(np.asarray(scale_bits, np.uint16).reshape(-1))
    if centered:
        s = (np.float32(1.0) + s).astype(np.float32)
    return np.broadcast_to(s, (d,)) if s.size == 1 else s


def row_sumsq(x: np.ndarray) -> np.ndarray:
    """Sum of squares of each row of a [rows, d] f32 array in the kernel's fixed order."""
    rows, d = x.shape
    nch = -(-d // 8)
    rounds = -(-nch // 32)
    xp = np.zeros((rows, rounds * 32 * 8), np.float32)
    xp[:, :d] = x
    xc = xp.reshape(rows, rounds, 32, 8)
    acc = np.zeros((rows, 32), np.float32)
    for i in range(rounds):
        for j in range(8):
            v = xc[:, i, :, j]
            acc = (acc + (v * v).astype(np.float32)).astype(np.float32)
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        acc = (acc + acc[:, lanes ^ o]).astype(np.float32)
    return acc[:, 0]


def rmsnorm(x_bits: np.ndarray, scale_bits=None, centered: bool = False, eps: float = 1e-6):
    """(y bf16 bits [rows, d], rstd f32 [rows]) for x given as bf16 bits [rows, d]."""
    x = bf16_bits_to_f32(np.asarray(x_bits, np.uint16))
    d = x.shape[-1]
    ss = row_sumsq(x)
    with np.errstate(divide="ignore", invalid="ignore"):
        var = (ss / np.float32(d)).astype(np.float32)
        r = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    w = _weight(scale_bits, centered, d)
    y = ((x * r[:, None]).astype(np.float32) * w[None, :]).astype(np.float32)
    return f32_to_bf16_bits(y), r


def rmsnorm_quant(x_bits, scale_bits=None, centered=False, eps=1e-6, fmt: int = 0, fast: bool = False):
    """RMSNorm followed by the per-tensor fp8 recipe on its output: (codes, amax, inv, y, rstd).
    fast: the ml_dtypes-backed cast (same codes; see fp8.quantize_bits)."""
    y, r = rmsnorm(x_bits, scale_bits, centered, eps)
    codes, amax, inv = quantize_bits(y.reshape(-1), fmt, fast=fast)
    return codes.reshape(y.shape), amax, inv, y, r


def rmsnorm_backward(x_bits, scale_bits, centered, rstd, dy_bits):
    """Float64 derivative of y = x * r * w with r = (mean(x^2) + eps)^-1/2 (r from the forward):
    dx = r w g - x r^3 sum(g w x) / d; dw = sum over rows of g x r (summed over the row for a
    one-element scale).  Returns (dx f64, dw f64 or None)."""
    x = bf16_bits_to_f32(np.asarray(x_bits, np.uint16)).astype(np.float64)
    g = bf16_bits_to_f32(np.asarray(dy_bits, np.uint16)).astype(np.float64)
    d = x.shape[-1]
    w = _weight(scale_bits, centered, d).astype(np.float64)
    r = np.asarray(rstd, np.float64)[:, None]
    a = (g * w * x).sum(axis=-1, keepdims=True)
    dx = r * w * g - x * (r ** 3) * a / d
    dw = None
    if scale_bits is not None:
        per = (g * x * r).sum(axis=0)
        dw = per if np.asarray(scale_bits).size > 1 else np.array([per.sum()])
    return dx, dw
