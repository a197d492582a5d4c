"""Restatement of the FP8 Einsum / GMLP path on the CPU (oracle; test infrastructure only).

Every tensor crosses this module as numpy arrays: bf16 tensors as uint16 bit patterns,
fp8 tensors as uint8 codes.  Contractions use np.einsum / np.matmul on the dequantised
operands (exact fp8 values) with the accumulation dtype the caller picks (float64 for
parity checks, float32 for the timed CPU baseline), then apply the product of the two
inverse scales in float32 and round to bf16.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import fp8 as fp8mod
from .fp8 import (E4M3, E5M2, amax_bits, bf16_bits_to_f32, f32_to_bf16_bits, fp8_to_f64, quantize_bits,
                  round_bf16)


@dataclass
class Q:
    """An fp8 tensor: codes, format, amax and inverse scale."""
    codes: np.ndarray
    fmt: int
    amax: np.float32
    inv: np.float32

    def deq(self, dtype=np.float64) -> np.ndarray:
        """Exact values of the codes (memoised per dtype: weights are reused in a step)."""
        cache = self.__dict__.setdefault("_deq", {})
        key = np.dtype(dtype).str
        if key not in cache:
            if fp8mod.THREADED and np.dtype(dtype) == np.float32:
                cache[key] = fp8mod.fp8_to_f32_threaded(self.codes, self.fmt)
            else:
                cache[key] = fp8_to_f64(self.codes, self.fmt).astype(dtype, copy=False)
        return cache[key]


# Module-wide switch: True makes every quantisation use the ml_dtypes-backed cast (same
# codes, verified by the tests) so that the oracle can be timed as the CPU baseline.
FAST_CAST = False


def quant(x_bits: np.ndarray, fmt: int, amax: np.float32 | None = None) -> Q:
    codes, a, inv = quantize_bits(x_bits, fmt, amax, fast=FAST_CAST)
    return Q(codes, fmt, a, inv)


def _scale_out(acc: np.ndarray, alpha: np.float32) -> np.ndarray:
    """acc * alpha in float32, as the GEMM epilogue does."""
    with np.errstate(over="ignore", invalid="ignore"):
        return acc.astype(np.float32) * np.float32(alpha)


def alpha_of(a: Q, b: Q) -> np.float32:
    with np.errstate(over="ignore", invalid="ignore"):
        return np.float32(a.inv) * np.float32(b.inv)


def gemm(a: Q, b: Q, a_expr: str, b_expr: str, out_expr: str, acc=np.float64, out_f32=False) -> np.ndarray:
    """bf16(einsum(deq(a), deq(b)) * inv_a * inv_b); returns bf16 bits (or f32)."""
    acc_v = np.einsum(f"{a_expr},{b_expr}->{out_expr}", a.deq(acc), b.deq(acc), optimize=True)
    y = _scale_out(acc_v, alpha_of(a, b))
    return y if out_f32 else f32_to_bf16_bits(y)


# ----------------------------------------------------------------------------- Einsum
def einsum_fp8(expr: str, x_bits: np.ndarray, w_bits: np.ndarray, fwd_fmt: int = E4M3, acc=np.float64):
    """FP8 mode of Einsum.__call__ (ueaj/model/einsum.py:233-251): quantise x and w per
    tensor, contract with the layer's own expression string, bf16 output."""
    lhs, out_expr = expr.split("->")
    x_expr, w_expr = lhs.split(",")
    qx, qw = quant(x_bits, fwd_fmt), quant(w_bits, fwd_fmt)
    return gemm(qx, qw, x_expr, w_expr, out_expr, acc), qx, qw


def einsum_fp8_backward(expr: str, qx: Q, qw: Q, dy_bits: np.ndarray, bwd_fmt: int = E5M2, acc=np.float64):
    """The two contractions JAX derives for the einsum's backward, with the incoming
    gradient cast per tensor to e5m2 (custom_astype backward, ueaj/utils/gradutils.py:46-51)."""
    lhs, out_expr = expr.split("->")
    x_expr, w_expr = lhs.split(",")
    qd = quant(dy_bits, bwd_fmt)
    dx = gemm(qd, qw, out_expr, w_expr, x_expr, acc)
    dw = gemm(qx, qd, x_expr, out_expr, w_expr, acc)
    return dx, dw


# ----------------------------------------------------------------------------- GMLP
def sigmoid32(g: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (np.float32(1.0) / (np.float32(1.0) + np.exp(-g.astype(np.float32)))).astype(np.float32)


def swiglu(u_bits: np.ndarray, g_bits: np.ndarray) -> np.ndarray:
    """h = up * swish(gate) (ueaj/model/mlp.py:103,107; nnx.swish(g) = g * sigmoid(g)),
    computed in float32 from the bf16 Einsum outputs, rounded to bf16."""
    u, g = bf16_bits_to_f32(u_bits), bf16_bits_to_f32(g_bits)
    return f32_to_bf16_bits(u * (g * sigmoid32(g)))


def dswiglu(dh: np.ndarray, u_bits: np.ndarray, g_bits: np.ndarray):
    """Autodiff of h = u * g * sigmoid(g): dU = dH * swish(g),
    dG = dH * u * sigmoid(g) * (1 + g * (1 - sigmoid(g))); dH rounded to bf16 first."""
    dh = round_bf16(dh)
    u, g = bf16_bits_to_f32(u_bits), bf16_bits_to_f32(g_bits)
    sg = sigmoid32(g)
    du = dh * (g * sg)
    dg = (dh * u) * (sg * (np.float32(1.0) + g * (np.float32(1.0) - sg)))
    return f32_to_bf16_bits(du), f32_to_bf16_bits(dg)


def gmlp_forward(x_bits: np.ndarray, wf_bits, wd_bits, acc=np.float64):
    """GMLP.__call__ (ueaj/model/mlp.py:100-115) with both Einsums in FP8.

    x [T, d], wf [2, d, h] (index 0 = up, 1 = gate), wd [h, d]; all bf16 bit patterns.
    wf / wd may also be given already quantised (Q), as one training step reuses them."""
    qx = quant(x_bits, E4M3)
    qwf = wf_bits if isinstance(wf_bits, Q) else quant(wf_bits, E4M3)
    acc_ug = np.einsum("td,idh->ith", qx.deq(acc), qwf.deq(acc), optimize=True)
    ug = f32_to_bf16_bits(_scale_out(acc_ug, alpha_of(qx, qwf)))
    hid = swiglu(ug[0], ug[1])
    qh = quant(hid, E4M3, amax_bits(hid))
    qwd = wd_bits if isinstance(wd_bits, Q) else quant(wd_bits, E4M3)
    y = gemm(qh, qwd, "th", "hd", "td", acc)
    return y, dict(qx=qx, qwf=qwf, ug=ug, h=hid, qh=qh, qwd=qwd)


def gmlp_backward(dy_bits: np.ndarray, saved: dict, acc=np.float64):
    """Backward of gmlp_forward: e5m2 output gradient, four contractions, gating backward."""
    qx, qwf, ug, qh, qwd = saved["qx"], saved["qwf"], saved["ug"], saved["qh"], saved["qwd"]
    qdy = quant(dy_bits, E5M2)
    dh = _scale_out(np.einsum("td,hd->th", qdy.deq(acc), qwd.deq(acc), optimize=True), alpha_of(qdy, qwd))
    du, dg = dswiglu(dh, ug[0], ug[1])
    dug = np.stack([du, dg])
    dwd = gemm(qh, qdy, "th", "td", "hd", acc)
    qdug = quant(dug, E5M2, amax_bits(dug))
    dx = gemm(qdug, qwf, "ith", "idh", "td", acc)
    dwf = gemm(qx, qdug, "td", "ith", "idh", acc)
    return dict(dx=dx, dwf=dwf, dwd=dwd, dug=dug, qdy=qdy, qdug=qdug)


# ----------------------------------------------------------------------------- inputs
def bf16_normal(rng: np.random.Generator, shape, std: float = 1.0) -> np.ndarray:
    """Seeded N(0, std^2) samples rounded to bf16 (bit patterns)."""
    return f32_to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * np.float32(std))
