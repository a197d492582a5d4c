"""The RoPE / attention oracle (oracle/attention.py) on the CPU: RoPE against the float64 rotation
and its transpose, the attention against a float64 softmax attention without the kernels' bf16
storage points, and the mask semantics (causality, segments, padding)."""
import numpy as np

from oracle import attention as oa
from oracle.fp8 import bf16_bits_to_f32, f32_to_bf16_bits
from oracle.path import bf16_normal


def test_rope_rotation_and_transpose():
    rng = np.random.default_rng(0)
    x = bf16_normal(rng, (2, 16, 3, 8))
    s, c = oa.rope_tables(np.arange(16), 8, 10000.0)
    y = bf16_bits_to_f32(oa.rope_apply(x, s, c))
    xf = bf16_bits_to_f32(x).astype(np.float64)
    s3, c3 = s[None, :, None, :].astype(np.float64), c[None, :, None, :].astype(np.float64)
    ref = np.concatenate([xf[..., :4] * c3 - xf[..., 4:] * s3, xf[..., 4:] * c3 + xf[..., :4] * s3], -1)
    np.testing.assert_allclose(y, ref, rtol=2 ** -7, atol=1e-2)
    back = bf16_bits_to_f32(oa.rope_apply(f32_to_bf16_bits(y), s, c, inverse=True))
    np.testing.assert_allclose(back, xf, rtol=2e-2, atol=2e-2)  # rotation then its transpose


def _naive(q, k, v, vis, scale):
    b, n, hi, dh = q.shape
    grp = hi // k.shape[2]
    out = np.zeros_like(q)
    for bi in range(b):
        for g in range(hi):
            s = scale * q[bi, :, g] @ k[bi, :, g // grp].T
            s = np.where(vis[bi], s, -np.inf)
            m = np.max(s, axis=1, keepdims=True)
            e = np.where(vis[bi], np.exp(s - np.where(np.isfinite(m), m, 0)), 0)
            t = e.sum(1, keepdims=True)
            out[bi, :, g] = np.where(t > 0, e / np.where(t > 0, t, 1), 0) @ v[bi, :, g // grp]
    return out


def test_attention_oracle_against_float64_and_mask_semantics():
    rng = np.random.default_rng(1)
    b, n, h, grp, dh = 2, 24, 2, 2, 16
    q = bf16_normal(rng, (b, n, h * grp, dh))
    k = bf16_normal(rng, (b, n, h, dh))
    v = bf16_normal(rng, (b, n, h, dh))
    seg = np.zeros((b, n), np.int64)
    seg[0, 10:] = 1          # two documents in sequence 0
    seg[1, 20:] = -1         # padding at the end of sequence 1
    pos = np.broadcast_to(np.arange(n), (b, n))
    out, P = oa.attention_forward(q, k, v, seg, seg, pos, pos, 0.25)
    vis = np.stack([oa._visible(seg[i], seg[i], pos[i], pos[i]) for i in range(b)])
    ref = _naive(*(bf16_bits_to_f32(t).astype(np.float64) for t in (q, k, v)), vis, 0.25)
    got = bf16_bits_to_f32(out)
    np.testing.assert_allclose(got, ref, atol=2e-2 * np.abs(ref).max())
    assert (got[1, 20:] == 0).all()                        # padding rows see nothing
    np.testing.assert_array_equal(P[0][:, :10, 10:], 0)    # document 0 never sees document 1
    assert np.triu(P[0, 0], 1).max() == 0                  # causal
    # a change in document 1 leaves document 0's outputs unchanged
    k2 = k.copy()
    k2[0, 15] = bf16_normal(rng, (h, dh))
    out2, _ = oa.attention_forward(q, k2, v, seg, seg, pos, pos, 0.25)
    np.testing.assert_array_equal(bf16_bits_to_f32(out2)[0, :10], got[0, :10])
