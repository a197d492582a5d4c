"""RoPE and softmax attention restated on the CPU (oracle; test infrastructure only).

Follows ueaj/model/rope.py:10-104 (compute_rope_embedding: angle = position * 1 / theta^(j / half)
in f32, sin / cos rounded to bf16; _apply_rope: (x1 c - x2 s, x2 c + x1 s) on bf16 values with each
operation rounded to bf16) and the flash_attention call of ueaj/model/soft_attn.py:186-196, whose
library (kvax 0.1.2, requirements.txt:35) is not installable here; its published semantics are
restated: softmax(scale * Q K^T) V per query head over the keys p' <= p of the same non-negative
segment (a row that sees nothing outputs 0), query head (h, i) with key/value head h.  Parity with
kvax itself is unpinned.

attention_forward / attention_backward follow the kernels' storage points so the GPU can be held
to the GEMM bar: scores accumulated in float64 and rounded to f32, scale * s in f32, softmax in
float64 then P rounded to bf16, O = P V accumulated in float64 and rounded to bf16; backward
dP = dO V^T (f32), D = rowsum(dO * O), dS = bf16(scale * P * (dP - D)), dQ = dS K, dK = sum over
the group of dS^T Q, dV = sum over the group of P^T dO (float64, rounded to bf16).
"""
from __future__ import annotations

import numpy as np

from .fp8 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def rope_inv_freq(rope_d: int, theta: float) -> np.ndarray:
    half = rope_d // 2
    e = (np.arange(half, dtype=np.float32) / np.float32(half)).astype(np.float32)
    return (np.float32(1.0) / np.power(np.float32(theta), e).astype(np.float32)).astype(np.float32)


def rope_tables(pos: np.ndarray, rope_d: int, theta: float):
    """(sin, cos) as f32 values of the bf16 tables, shape pos.shape + (rope_d / 2,)."""
    a = (np.asarray(pos, np.float32)[..., None] * rope_inv_freq(rope_d, theta)).astype(np.float32)
    return round_bf16(np.sin(a).astype(np.float32)), round_bf16(np.cos(a).astype(np.float32))


def rope_apply(x_bits: np.ndarray, sin: np.ndarray, cos: np.ndarray, inverse: bool = False) -> np.ndarray:
    """x bf16 bits [b, n, ..., d]; sin / cos [n, half] or [b, n, half] -> bf16 bits."""
    x = bf16_bits_to_f32(x_bits)
    half = x.shape[-1] // 2
    extra = x.ndim - 3
    if sin.ndim == 2:
        sin = sin[None]
        cos = cos[None]
    shape = sin.shape[:2] + (1,) * extra + (half,)
    s, c = sin.reshape(shape), cos.reshape(shape)
    x1, x2 = x[..., :half], x[..., half:]
    r = round_bf16
    if not inverse:
        o1 = (r((x1 * c).astype(np.float32)) - r((x2 * s).astype(np.float32))).astype(np.float32)
        o2 = (r((x2 * c).astype(np.float32)) + r((x1 * s).astype(np.float32))).astype(np.float32)
    else:
        o1 = (r((x1 * c).astype(np.float32)) + r((x2 * s).astype(np.float32))).astype(np.float32)
        o2 = (r((x2 * c).astype(np.float32)) - r((x1 * s).astype(np.float32))).astype(np.float32)
    return f32_to_bf16_bits(np.concatenate([o1, o2], axis=-1))


def _visible(qseg, kseg, qpos, kpos):
    """[n, n] boolean: query p sees key p'."""
    return (qseg[:, None] >= 0) & (kseg[None, :] == qseg[:, None]) & (kpos[None, :] <= qpos[:, None])


def attention_forward(q_bits, k_bits, v_bits, qseg=None, kseg=None, qpos=None, kpos=None, scale=1.0):
    """q [b, n, hi, d], k / v [b, n, h, d] bf16 bits -> (out bits [b, n, hi, d], P f32 values)."""
    q, k, v = (bf16_bits_to_f32(t).astype(np.float64) for t in (q_bits, k_bits, v_bits))
    b, n, hi, dh = q.shape
    h = k.shape[2]
    grp = hi // h
    qseg = np.zeros((b, n), np.int64) if qseg is None else np.asarray(qseg)
    kseg = qseg if kseg is None else np.asarray(kseg)
    qpos = np.broadcast_to(np.arange(n), (b, n)) if qpos is None else np.asarray(qpos)
    kpos = qpos if kpos is None else np.asarray(kpos)
    out = np.zeros((b, n, hi, dh), np.float64)
    P = np.zeros((b, hi, n, n), np.float32)
    for bi in range(b):
        vis = _visible(qseg[bi], kseg[bi], qpos[bi], kpos[bi])
        for g in range(hi):
            kh = g // grp
            s = (q[bi, :, g] @ k[bi, :, kh].T).astype(np.float32)
            s = (s * np.float32(scale)).astype(np.float32).astype(np.float64)
            s = np.where(vis, s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0)
            e = np.where(vis, np.exp(s - m), 0.0)
            tot = e.sum(axis=1, keepdims=True)
            p = round_bf16(np.where(tot > 0, e / np.where(tot > 0, tot, 1.0), 0.0).astype(np.float32))
            P[bi, g] = p
            out[bi, :, g] = p.astype(np.float64) @ v[bi, :, kh]
    return f32_to_bf16_bits(out.astype(np.float32)), P


def attention_backward(dout_bits, out_bits, P, q_bits, k_bits, v_bits, scale=1.0):
    """-> (dq, dk, dv) as f64 arrays (the kernels round them to bf16)."""
    q, k, v, o, go = (bf16_bits_to_f32(t).astype(np.float64) for t in (q_bits, k_bits, v_bits, out_bits, dout_bits))
    b, n, hi, dh = q.shape
    h = k.shape[2]
    grp = hi // h
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for bi in range(b):
        for g in range(hi):
            kh = g // grp
            p = P[bi, g].astype(np.float64)
            dp = (go[bi, :, g] @ v[bi, :, kh].T).astype(np.float32).astype(np.float64)
            D = (go[bi, :, g] * o[bi, :, g]).sum(axis=1, keepdims=True)
            ds = round_bf16((np.float32(scale) * (p * (dp - D))).astype(np.float32)).astype(np.float64)
            dq[bi, :, g] = ds @ k[bi, :, kh]
            dk[bi, :, kh] += ds.T @ q[bi, :, g]
            dv[bi, :, kh] += p.T @ go[bi, :, g]
    return dq, dk, dv
