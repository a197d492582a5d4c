"""Next-token cross-entropy on the lm_head logits, restated on the CPU (oracle; test
infrastructure only).

Follows, relative to the macrogpt-jax repository:
  * ntp_loss_mask / ntp_args  ueaj/opt/next_token_loss.py:13-97 (last position masked; positions
    whose next token is padding or crosses a document boundary masked; targets shifted by one);
  * chunked_softmax_cross_entropy  ueaj/opt/next_token_loss.py:99-174: per-token
    optax.softmax_cross_entropy_with_integer_labels(logits, targets) * mask, i.e.
    logsumexp(logits) - logits[target], with the target logit gathered by jnp.take_along_axis
    (negative indices count from the end; out-of-range indices read NaN in its fill mode);
  * LlamaModel.get_logits  ueaj/model/model.py:140-165: final norm, lm_head Einsum "bnd,dv->bnv",
    then 15 * tanh(logits / 15) when head_cap == 'tanh', evaluated on bf16 values with each
    operation rounded to bf16;
  * the derivative JAX takes of the loss: dl = g * (softmax - onehot), times tanh'(l / 15) for the
    capped head, with g = upstream gradient * mask.

The FP8 lm_head quantises its input, weight and the incoming logit gradient per tensor like every
FP8 Einsum of this package (path.py).  The scale of the logit gradient comes from per-row results
(amax = max_r |g_r| * (1 - softmax_r[label_r]), the largest |dl| of each row sits at its label),
which equals the tensor's own amax in exact arithmetic; xent_backward restates that choice and the
kernel's f32 operation order.  Parity against the reference's JAX output is unpinned (JAX cannot
run here); where the reference leaves the arithmetic to XLA (the logsumexp's reduction order, the
tanh approximation), the loss is compared within a tolerance.
"""
from __future__ import annotations

import numpy as np

from . import norm as onorm
from . import path as _path
from .fp8 import (E4M3, E5M2, bf16_bits_to_f32, f32_to_bf16_bits, f32_to_fp8, f32_to_fp8_fast, round_bf16,
                  scale_from_amax)
from .path import Q, gemm, quant

BF16 = 2  # unquantised gradient output


def ntp_loss_mask(inputs, document_ids=None, pad_token_id=None, loss_mask=None) -> np.ndarray:
    """ueaj/opt/next_token_loss.py:13-58 on [batch, seq] integer arrays."""
    inputs = np.asarray(inputs)
    mask = np.ones(inputs.shape[:2], np.int32)
    mask[:, -1] = 0
    if loss_mask is not None:
        mask = mask * np.asarray(loss_mask).astype(np.int32)
    if pad_token_id is not None:
        mask[:, :-1] *= (inputs[:, 1:] != pad_token_id)
    if document_ids is not None:
        doc = np.asarray(document_ids)
        mask[:, :-1] *= (doc[:, :-1] == doc[:, 1:])
    return mask


def ntp_args(inputs, document_ids=None, pad_token_id=None, loss_mask=None):
    """ueaj/opt/next_token_loss.py:61-97: (targets, mask); targets[:, i] = inputs[:, i + 1], the last
    position keeps its own token (masked anyway)."""
    inputs = np.asarray(inputs)
    mask = ntp_loss_mask(inputs, document_ids, pad_token_id, loss_mask)
    targets = inputs.copy()
    targets[:, :-1] = inputs[:, 1:]
    return targets, mask


def soft_cap(logit_bits: np.ndarray, cap: float = 15.0) -> np.ndarray:
    """cap * tanh(l / cap) on bf16 logits with bf16 rounding after each operation (f32 inside)."""
    l = bf16_bits_to_f32(logit_bits)
    c = np.float32(cap)
    t1 = round_bf16((l / c).astype(np.float32))
    t2 = round_bf16(np.tanh(t1).astype(np.float32))
    return f32_to_bf16_bits((c * t2).astype(np.float32))


def label_cols(labels, V: int) -> np.ndarray:
    """Column of each label (negative counts from the end), -1 where outside [-V, V)."""
    lab = np.asarray(labels, np.int64)
    col = np.where(lab < 0, lab + V, lab)
    return np.where((col >= 0) & (col < V), col, -1)


def xent_rows(logit_bits: np.ndarray, labels, mask=None):
    """Per row of bf16 logits [rows, V]: (lse, loss, qrow) as f32.  lse = logsumexp in f64;
    loss = (lse - c[label]) * mask (NaN without a label column); qrow = 1 - exp(c[label] - lse)
    (float64 here; the kernels compute it with softmax_p's f32 operations)."""
    c = bf16_bits_to_f32(np.asarray(logit_bits, np.uint16)).astype(np.float64)
    rows, V = c.shape
    with np.errstate(invalid="ignore", over="ignore"):
        M = c.max(axis=1) if V else np.zeros(rows)
        lse = M + np.log(np.exp(c - M[:, None]).sum(axis=1))
    col = label_cols(labels, V)
    r = np.arange(rows)
    cl = np.where(col >= 0, c[r, np.maximum(col, 0)], np.nan)
    mk = np.ones(rows) if mask is None else np.asarray(mask, np.float64).reshape(-1)
    with np.errstate(invalid="ignore"):
        loss = (lse - cl) * mk
        qrow = np.where(col >= 0, 1.0 - np.exp(cl - lse), 1.0)
    return lse.astype(np.float32), loss.astype(np.float32), qrow.astype(np.float32)


LOG2E = np.float32(1.4426950408889634)


def softmax_p(c: np.ndarray, lse: np.ndarray) -> np.ndarray:
    """p = 2^(c * log2 e - lse * log2 e): the product with log2 e and the sum rounded once (the
    kernel's FMA; float64 holds the f32 product exactly), exp2 in f32."""
    nl2 = (np.asarray(lse, np.float32) * -LOG2E).astype(np.float32)
    x = (c.astype(np.float64) * np.float64(LOG2E) + nl2.astype(np.float64)[..., None]).astype(np.float32)
    with np.errstate(over="ignore", under="ignore"):
        return np.exp2(x).astype(np.float32)


def xent_backward(logit_bits: np.ndarray, labels, mask, lse, qrow, dloss=None, cap: float = 0.0, fmt: int = E5M2):
    """dlogits with the kernel's f32 operation order: p = softmax_p(c, lse); d = p - [j == label];
    the row factor w = g (bf16 output) or g * s (fp8), g = dloss * mask; v = d * w; with a cap,
    v *= 1 - (c * (1 / cap))^2.  fmt BF16: bf16 bits of v.  fp8: amax = max_r |g_r| * qrow_r,
    s = FMAX / amax, codes = fp8(v); returns (codes, amax, inv_scale)."""
    c = bf16_bits_to_f32(np.asarray(logit_bits, np.uint16))
    rows, V = c.shape
    lse = np.asarray(lse, np.float32).reshape(rows)
    g = np.ones(rows, np.float32) if dloss is None else np.asarray(dloss, np.float32).reshape(rows)
    mk = np.ones(rows, np.float32) if mask is None else np.asarray(mask).astype(np.float32).reshape(rows)
    ge = (g * mk).astype(np.float32)
    amax = s = inv = None
    if fmt == BF16:
        w = ge
    else:
        qr = np.asarray(qrow, np.float32).reshape(rows)
        with np.errstate(invalid="ignore"):
            per = (np.abs(ge) * qr).astype(np.float32)
        amax = np.float32(0.0) if rows == 0 else (np.float32(np.nan) if np.isnan(per).any() else per.max())
        s = scale_from_amax(amax, fmt)
        with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
            inv = np.float32(np.float32(1.0) / s)
            w = (ge * s).astype(np.float32)
    with np.errstate(over="ignore", invalid="ignore"):
        p = softmax_p(c, lse)
        col = label_cols(labels, V)
        r = np.nonzero(col >= 0)[0]
        p[r, col[r]] = (p[r, col[r]] - np.float32(1.0)).astype(np.float32)
        v = (p * w[:, None]).astype(np.float32)
        if cap > 0:
            t = (c * np.float32(1.0 / np.float32(cap))).astype(np.float32)
            v = (v * (np.float32(1.0) - (t * t).astype(np.float32)).astype(np.float32)).astype(np.float32)
    if fmt == BF16:
        return f32_to_bf16_bits(v)
    with np.errstate(over="ignore", invalid="ignore"):
        cast = f32_to_fp8_fast if _path.FAST_CAST else f32_to_fp8  # same codes (fp8.py)
        codes = cast(v, fmt)
    return codes, np.float32(amax), inv


def head_forward(x_bits, scale_bits, centered, eps, w_bits, labels, mask=None, cap: float = 0.0, acc=np.float64):
    """Final RMSNorm -> FP8 lm_head "bnd,dv->bnv" -> (soft cap) -> per-token masked loss.
    x [T, d], w [d, V] as bf16 bits.  Returns (loss f32 [T], saved dict)."""
    codes, amax, inv, y, rstd = onorm.rmsnorm_quant(x_bits, scale_bits, centered, eps, E4M3, fast=_path.FAST_CAST)
    qx = Q(codes, E4M3, amax, inv)
    qw = w_bits if isinstance(w_bits, Q) else quant(w_bits, E4M3)
    logits = gemm(qx, qw, "td", "dv", "tv", acc)
    if cap > 0:
        logits = soft_cap(logits, cap)
    lse, loss, qrow = xent_rows(logits, labels, mask)
    return loss, dict(qx=qx, qw=qw, logits=logits, lse=lse, qrow=qrow, rstd=rstd, y=y)


def head_backward(dloss, saved, x_bits, scale_bits, centered, labels, mask=None, cap: float = 0.0, acc=np.float64):
    """Backward of head_forward: e5m2 dlogits, dX = dL W^T, dW = X^T dL (FP8, bf16 out), then the
    norm's backward.  Returns dict(dx f64, dscale f64 or None, dw bits, dxn bits, qd)."""
    codes, amax, inv = xent_backward(saved["logits"], labels, mask, saved["lse"], saved["qrow"], dloss, cap, E5M2)
    qd = Q(codes, E5M2, amax, inv)
    dxn = gemm(qd, saved["qw"], "tv", "dv", "td", acc)
    dw = gemm(saved["qx"], qd, "td", "tv", "dv", acc)
    dx, dscale = onorm.rmsnorm_backward(x_bits, scale_bits, centered, saved["rstd"], dxn)
    return dict(dx=dx, dscale=dscale, dw=dw, dxn=dxn, qd=qd)
