"""The cross-entropy oracle (oracle/xent.py) and the host-side mask/target logic, on the CPU.

Known answers come from the reference's own docstring examples (ueaj/opt/next_token_loss.py:40-45,
86-92 and its __main__ block, 176-181); the loss and its gradient are checked against independent
float64 formulas."""
import numpy as np
import pytest
import torch

from oracle import xent as ox
from oracle.fp8 import E4M3, E5M2, FMAX, bf16_bits_to_f32, f32_to_bf16_bits, fp8_to_f64
from oracle.path import bf16_normal


def test_ntp_known_answers():
    targets, mask = ox.ntp_args(np.array([[1, 2, 3, 4, 5]]))
    assert targets.tolist() == [[2, 3, 4, 5, 5]]
    assert mask.tolist() == [[1, 1, 1, 1, 0]]
    assert ox.ntp_loss_mask(np.array([[1, 2, 3, 0, 0]]), pad_token_id=0).tolist() == [[1, 1, 0, 0, 0]]
    # __main__ block: tokens [[1,2,3,4,5,0]], documents [[1,1,1,2,2,2]], pad 0
    t, m = ox.ntp_args(np.array([[1, 2, 3, 4, 5, 0]]), np.array([[1, 1, 1, 2, 2, 2]]), 0)
    assert t.tolist() == [[2, 3, 4, 5, 0, 0]]
    assert m.tolist() == [[1, 1, 0, 1, 0, 0]]


def test_host_ntp_matches_oracle():
    from macrogpt_jax_b200 import next_token_loss as ntl
    rng = np.random.default_rng(3)
    inputs = rng.integers(0, 6, (4, 33))
    docs = np.cumsum(rng.random((4, 33)) < 0.1, axis=1)
    lm = rng.integers(0, 2, (4, 33))
    for kw in ({}, dict(pad_token_id=0), dict(document_ids=docs), dict(loss_mask=lm),
               dict(document_ids=docs, pad_token_id=0, loss_mask=lm)):
        t_ref, m_ref = ox.ntp_args(inputs, **kw)
        tkw = {k: (torch.from_numpy(v) if isinstance(v, np.ndarray) else v) for k, v in kw.items()}
        t, m = ntl.ntp_args(torch.from_numpy(inputs), **tkw)
        assert np.array_equal(t.numpy(), t_ref)
        assert np.array_equal(m.numpy(), m_ref)


def _logits(rng, rows, V, std=3.0):
    return bf16_normal(rng, (rows, V), std)


def test_xent_rows_against_logsumexp():
    from scipy.special import logsumexp
    rng = np.random.default_rng(0)
    lb = _logits(rng, 37, 301)
    labels = rng.integers(-301, 301, 37).astype(np.int32)
    labels[:3] = [301, -302, 10 ** 6]  # no column: NaN loss
    mask = rng.integers(0, 2, 37).astype(np.uint8)
    lse, loss, qrow = ox.xent_rows(lb, labels, mask)
    c = bf16_bits_to_f32(lb).astype(np.float64)
    ref = logsumexp(c, axis=1)
    np.testing.assert_allclose(lse, ref, rtol=1e-6)
    col = np.where(labels < 0, labels + 301, labels)
    for r in range(37):
        if r < 3:
            assert np.isnan(loss[r]) and qrow[r] == 1.0
            continue
        np.testing.assert_allclose(loss[r], (ref[r] - c[r, col[r]]) * mask[r], rtol=1e-6, atol=1e-6)
        np.testing.assert_allclose(qrow[r], 1.0 - np.exp(c[r, col[r]] - ref[r]), rtol=1e-5, atol=1e-7)


@pytest.mark.parametrize("cap", [0.0, 15.0])
def test_xent_backward_bf16_against_f64(cap):
    rng = np.random.default_rng(1)
    rows, V = 24, 130
    lb = _logits(rng, rows, V)
    if cap:
        lb = ox.soft_cap(lb, cap)
    labels = rng.integers(0, V, rows).astype(np.int32)
    mask = rng.integers(0, 2, rows).astype(np.uint8)
    dloss = rng.standard_normal(rows).astype(np.float32)
    lse, _, qrow = ox.xent_rows(lb, labels, mask)
    got = bf16_bits_to_f32(ox.xent_backward(lb, labels, mask, lse, qrow, dloss, cap, ox.BF16)).astype(np.float64)
    c = bf16_bits_to_f32(lb).astype(np.float64)
    p = np.exp(c - lse[:, None].astype(np.float64))
    p[np.arange(rows), labels] -= 1.0
    ref = (dloss * mask)[:, None] * p
    if cap:
        ref *= 1.0 - (c / cap) ** 2
    np.testing.assert_allclose(got, ref, rtol=2 ** -7, atol=1e-30)


@pytest.mark.parametrize("fmt", [E5M2, E4M3])
def test_xent_backward_fp8_scale_is_the_label_column(fmt):
    """amax from the row results equals max |dl| (the label column holds each row's largest
    |softmax - onehot|), so the largest code is +-FMAX and nothing overflows."""
    rng = np.random.default_rng(2)
    rows, V = 40, 257
    lb = _logits(rng, rows, V)
    labels = rng.integers(0, V, rows).astype(np.int32)
    dloss = rng.standard_normal(rows).astype(np.float32)
    lse, _, qrow = ox.xent_rows(lb, labels, None)
    codes, amax, inv = ox.xent_backward(lb, labels, None, lse, qrow, dloss, 0.0, fmt)
    v = bf16_bits_to_f32(ox.xent_backward(lb, labels, None, lse, qrow, dloss, 0.0, ox.BF16))
    assert np.isclose(amax, np.abs(v).max(), rtol=1e-2)
    deq = fp8_to_f64(codes, fmt)
    assert np.isfinite(deq).all()
    assert np.isclose(np.abs(deq).max(), FMAX[fmt], rtol=0.3)
    np.testing.assert_allclose(deq * inv, v, rtol=0.13 if fmt == E5M2 else 0.07, atol=float(amax) * 2e-5)


def test_xent_backward_degenerate_cases():
    lb = f32_to_bf16_bits(np.zeros((3, 4), np.float32))
    labels = np.array([0, 1, 9], np.int32)
    lse, loss, qrow = ox.xent_rows(lb, labels, None)
    np.testing.assert_allclose(lse, np.log(4.0), rtol=1e-7)
    assert np.isnan(loss[2]) and qrow[2] == 1.0
    codes, amax, inv = ox.xent_backward(lb, labels, np.zeros(3, np.uint8), lse, qrow, None, 0.0, E5M2)
    assert amax == 0 and inv == 1.0  # fully masked: amax 0 -> s = 1
    assert (fp8_to_f64(codes, E5M2) == 0).all()
    codes, amax, inv = ox.xent_backward(lb[:0], labels[:0], None, lse[:0], qrow[:0], None, 0.0, E5M2)
    assert codes.shape == (0, 4) and amax == 0 and inv == 1.0


def test_head_oracle_composes_the_quantised_contractions():
    """head_forward / head_backward against float64 contractions of the same quantised operands."""
    rng = np.random.default_rng(4)
    T, d, V = 20, 64, 96
    xb = bf16_normal(rng, (T, d))
    wb = bf16_normal(rng, (d, V), d ** -0.5)
    sb = bf16_normal(rng, (d,), 0.1)
    labels = rng.integers(0, V, T).astype(np.int32)
    loss, sv = ox.head_forward(xb, sb, True, 1e-6, wb, labels, None, 15.0)
    l64 = sv["qx"].deq() @ sv["qw"].deq() * (float(sv["qx"].inv) * float(sv["qw"].inv))
    l64 = 15.0 * np.tanh(l64 / 15.0)
    from scipy.special import logsumexp
    ref = logsumexp(l64, axis=1) - l64[np.arange(T), labels]
    np.testing.assert_allclose(loss, ref, atol=5e-2)
    g = ox.head_backward(np.ones(T, np.float32), sv, xb, sb, True, labels, None, 15.0)
    qd = g["qd"]
    dxn = qd.deq() @ sv["qw"].deq().T * (float(qd.inv) * float(sv["qw"].inv))
    dw = sv["qx"].deq().T @ qd.deq() * (float(sv["qx"].inv) * float(qd.inv))
    np.testing.assert_allclose(bf16_bits_to_f32(g["dxn"]), dxn, rtol=1e-2, atol=1e-6 * np.abs(dxn).max())
    np.testing.assert_allclose(bf16_bits_to_f32(g["dw"]), dw, rtol=1e-2, atol=1e-6 * np.abs(dw).max())
