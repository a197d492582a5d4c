"""Bit-level fp8 / bf16 arithmetic in numpy (oracle; test infrastructure only).

Formats (ml_dtypes 0.5.4 names, reference requirements.txt:38):
  float8_e4m3fn  1 sign, 4 exponent (bias 7), 3 mantissa; no inf; NaN = S.1111.111; max 448
  float8_e5m2    1 sign, 5 exponent (bias 15), 2 mantissa; inf = S.11111.00; max 57344
Casts from f32 round to nearest, ties to even, and do not saturate: e4m3fn values above
464 (and +-inf) become NaN with the input's sign; e5m2 values at or above 61440 become inf.
A NaN input becomes the positive NaN pattern (0x7F / 0x7E), the pattern a GPU's canonical
NaN maps to; ml_dtypes would keep the sign of a negative NaN.
"""
from __future__ import annotations

import numpy as np

E4M3, E5M2 = 0, 1
FMAX = {E4M3: 448.0, E5M2: 57344.0}
_MBITS = {E4M3: 3, E5M2: 2}
_BIAS = {E4M3: 7, E5M2: 15}


def _decode_table(fmt: int) -> np.ndarray:
    """float64 value of each of the 256 codes."""
    mb, bias = _MBITS[fmt], _BIAS[fmt]
    ebits = 7 - mb
    out = np.empty(256, dtype=np.float64)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> mb) & ((1 << ebits) - 1)
        m = code & ((1 << mb) - 1)
        if fmt == E4M3 and e == 15 and m == 7:
            v = np.nan
        elif fmt == E5M2 and e == 31:
            v = np.inf if m == 0 else np.nan
        elif e == 0:
            v = m * 2.0 ** (1 - bias - mb)
        else:
            v = (1.0 + m / (1 << mb)) * 2.0 ** (e - bias)
        out[code] = s * v
    return out


DECODE = {E4M3: _decode_table(E4M3), E5M2: _decode_table(E5M2)}
# Non-negative finite values in code order (codes 0x00.. are increasing in value).
_POS_FINITE = {f: DECODE[f][: (0x7F if f == E4M3 else 0x7C)] for f in (E4M3, E5M2)}


def fp8_to_f64(codes: np.ndarray, fmt: int) -> np.ndarray:
    return DECODE[fmt][np.asarray(codes, dtype=np.uint8)]


def f32_to_fp8(x: np.ndarray, fmt: int) -> np.ndarray:
    """Round-to-nearest-even cast of float32 values to fp8 codes (uint8)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x.astype(np.float64))
    sign = (np.signbit(x).astype(np.uint8)) << 7
    mb, bias = _MBITS[fmt], _BIAS[fmt]
    emin = 1 - bias
    finite = np.isfinite(a)
    safe = np.where(finite & (a > 0), a, 1.0)
    _, E = np.frexp(safe)  # safe = m * 2**E, m in [0.5, 1)
    e = np.maximum(E - 1, emin)
    quantum = np.ldexp(1.0, e - mb)
    v = np.rint(safe / quantum) * quantum  # np.rint rounds half to even; exact in float64
    v = np.where(a > 0, v, 0.0)
    limit = FMAX[fmt]
    over = finite & (v > limit)
    idx = np.searchsorted(_POS_FINITE[fmt], np.minimum(v, limit))
    codes = (idx.astype(np.uint8) | sign).astype(np.uint8)
    if fmt == E4M3:
        codes = np.where(over | np.isinf(a), np.uint8(0x7F) | sign, codes)
        codes = np.where(np.isnan(a), np.uint8(0x7F), codes)
    else:
        codes = np.where(over | np.isinf(a), np.uint8(0x7C) | sign, codes)
        codes = np.where(np.isnan(a), np.uint8(0x7E), codes)
    return codes.astype(np.uint8)


def f32_to_fp8_fast(x: np.ndarray, fmt: int) -> np.ndarray:
    """Same codes as f32_to_fp8, computed by ml_dtypes 0.5.4's C++ cast (the reference's
    pinned cast library) with NaN mapped to the positive pattern.  Used where the oracle is
    timed as the CPU baseline; tests check it equals f32_to_fp8."""
    import ml_dtypes

    x = np.asarray(x, dtype=np.float32)
    dt = ml_dtypes.float8_e4m3fn if fmt == E4M3 else ml_dtypes.float8_e5m2
    with np.errstate(invalid="ignore", over="ignore"):
        codes = x.astype(dt).view(np.uint8)
    nan = np.isnan(x)
    if nan.any():
        codes = np.where(nan, np.uint8(0x7F if fmt == E4M3 else 0x7E), codes)
    return codes


# ----------------------------------------------------------------------------- threaded passes
# THREADED = True routes the element-wise passes of the oracle through torch's multi-threaded
# CPU kernels (exact conversions: bf16 <-> f32, fp8 -> f32, and the RNE f32 -> bf16 rounding),
# for the CPU baseline, which times the oracle on all host cores.  Tensors holding a NaN take
# the numpy path, whose NaN handling is the specified one.  tests/test_oracle.py checks both
# paths give identical bits.
THREADED = False


def _torch():
    import torch
    return torch


def _bf16_bits_to_f32_threaded(bits: np.ndarray) -> np.ndarray:
    torch = _torch()
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).float().numpy()


def _f32_to_bf16_bits_threaded(x: np.ndarray):
    torch = _torch()
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    if bool(torch.isnan(t).any()):
        return None
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def fp8_to_f32_threaded(codes: np.ndarray, fmt: int) -> np.ndarray:
    """float32 values of fp8 codes (exact) through torch's fp8 decode."""
    torch = _torch()
    c = torch.from_numpy(np.ascontiguousarray(codes, dtype=np.uint8))
    return c.view(torch.float8_e4m3fn if fmt == E4M3 else torch.float8_e5m2).float().numpy()


# ----------------------------------------------------------------------------- bf16
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    if THREADED:
        return _bf16_bits_to_f32_threaded(bits)
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 (NaN stays NaN, quieted).

    For every non-NaN pattern b (at most 0xFF800000), b + 0x7FFF + 1 stays below 2**32,
    so the rounding add is done in uint32."""
    if THREADED:
        out = _f32_to_bf16_bits_threaded(x)
        if out is not None:
            return out
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32)
    r = (b >> 16) & np.uint32(1)
    r += b
    r += np.uint32(0x7FFF)
    out = (r >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = ((b[nan] >> 16) | np.uint32(0x40)).astype(np.uint16)
    return out


def round_bf16(x: np.ndarray) -> np.ndarray:
    """f32 values rounded to the nearest bf16, returned as f32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


# ----------------------------------------------------------------------------- recipe
def amax_bits(x_bits: np.ndarray) -> np.float32:
    """max |x| over bf16 bit patterns (sign cleared; NaN patterns sort above inf)."""
    b = np.asarray(x_bits, dtype=np.uint16).reshape(-1)
    if b.size == 0:
        return np.float32(0.0)
    m = np.uint32(int((b & 0x7FFF).max())) << 16
    return np.array([m], dtype=np.uint32).view(np.float32)[0]


F32_MAX = np.float32(np.finfo(np.float32).max)


def scale_from_amax(amax: np.float32, fmt: int) -> np.float32:
    """s = min(FMAX / amax, FLT_MAX); 1 for amax == 0; NaN for a NaN amax.

    The cap keeps s finite for amax below FMAX / FLT_MAX (still normal bf16 values), where the
    quotient overflows to inf and would turn every code non-finite (0 * inf = NaN)."""
    with np.errstate(over="ignore", divide="ignore", invalid="ignore"):
        if amax == 0:
            return np.float32(1.0)
        s = np.float32(FMAX[fmt]) / np.float32(amax)
        return s if np.isnan(s) else np.minimum(s, F32_MAX)


def quantize_bits(x_bits: np.ndarray, fmt: int, amax: np.float32 | None = None, fast: bool = False):
    """Per-tensor current scaling of a bf16 tensor given as bit patterns.

    Returns (codes uint8, amax f32, inv_scale f32)."""
    if amax is None:
        amax = amax_bits(x_bits)
    s = scale_from_amax(np.float32(amax), fmt)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        p = bf16_bits_to_f32(x_bits) * s  # float32 * float32, IEEE round to nearest
        inv = np.float32(1.0) / s
    cast = f32_to_fp8_fast if fast else f32_to_fp8
    return cast(p, fmt), np.float32(amax), np.float32(inv)
