"""RoPE (ufp8_rope_table / ufp8_rope) and the softmax attention (ufp8_attention_forward /
_backward) against the oracle (oracle/attention.py), and SoftmaxAttention / TransformerLayer end to
end.

Bars: RoPE with the kernel's own sin / cos tables bit-exact (the tables themselves: sinf / cosf
against numpy's f32 sin / cos, each rounded to bf16, may differ by one bf16 step in a few entries);
attention outputs and gradients at the GEMM bar of helpers.py (2e-2 of max, cosine 0.9999) against
the oracle's storage points (P may round one bf16 step apart where MUFU exp and float64 exp
straddle a rounding boundary)."""
import numpy as np
import pytest

from oracle import attention as oa
from oracle.fp8 import bf16_bits_to_f32
from oracle.path import bf16_normal

from helpers import bits_to_torch_bf16, compare, torch_bf16_to_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("pos_2d", [False, True])
def test_rope_against_oracle(cuda, pos_2d):
    import torch
    from macrogpt_jax_b200.attention import RoPE
    rng = np.random.default_rng(3)
    b, n, h, i, d = 2, 48, 3, 2, 128
    xb = bf16_normal(rng, (b, n, h, i, d))
    x = bits_to_torch_bf16(xb, cuda).requires_grad_(True)
    pos = rng.integers(0, 4096, (b, n)) if pos_2d else np.arange(n)
    rope = RoPE(rope_theta=10000.0, rope_d=d, value_dtype=torch.bfloat16)
    sin, cos = rope.compute_freqs(torch.from_numpy(pos).to(cuda))
    rs, rc = oa.rope_tables(pos, d, 10000.0)
    gs, gc = sin.float().cpu().numpy(), cos.float().cpu().numpy()
    assert (gs != rs).mean() <= 1e-2 and (gc != rc).mean() <= 1e-2
    assert np.abs(gs - rs).max() <= 2 ** -7 and np.abs(gc - rc).max() <= 2 ** -7
    y = rope(x, position_ids=torch.from_numpy(pos).to(cuda))
    assert np.array_equal(torch_bf16_to_bits(y), oa.rope_apply(xb, gs, gc))
    gb = bf16_normal(rng, (b, n, h, i, d))
    y.backward(bits_to_torch_bf16(gb, cuda))
    assert np.array_equal(torch_bf16_to_bits(x.grad), oa.rope_apply(gb, gs, gc, inverse=True))


def _segments(b, n, rng):
    seg = np.zeros((b, n), np.int32)
    if b > 1:
        seg[1, n // 3:] = 1
        seg[1, n - n // 8:] = -1  # padding at the end
    return seg


@pytest.mark.parametrize("b,n,h,grp,dh", [(2, 128, 2, 2, 64), (1, 256, 4, 1, 128), (2, 136, 1, 4, 128)])
def test_attention_against_oracle(cuda, b, n, h, grp, dh):
    import torch
    from macrogpt_jax_b200.attention import softmax_attention
    rng = np.random.default_rng(b * n + h + grp + dh)
    qb = bf16_normal(rng, (b, n, h * grp, dh))
    kb = bf16_normal(rng, (b, n, h, dh))
    vb = bf16_normal(rng, (b, n, h, dh))
    seg = _segments(b, n, rng)
    pos = np.broadcast_to(np.arange(n, dtype=np.int32), (b, n)).copy()
    scale = dh ** -0.5
    q, k, v = (bits_to_torch_bf16(t, cuda).requires_grad_(True) for t in (qb, kb, vb))
    segt, post = torch.from_numpy(seg).to(cuda), torch.from_numpy(pos).to(cuda)
    out = softmax_attention(q, k, v, post, segt, post, segt, scale=scale)
    gob = bf16_normal(rng, (b, n, h * grp, dh))
    out.backward(bits_to_torch_bf16(gob, cuda))
    torch.cuda.synchronize()
    ro, P = oa.attention_forward(qb, kb, vb, seg, seg, pos, pos, scale)
    got = bf16_bits_to_f32(torch_bf16_to_bits(out))
    compare(got, bf16_bits_to_f32(ro))
    if b > 1:
        assert (got[1, n - n // 8:] == 0).all()  # padding rows see nothing
    dq, dk, dv = oa.attention_backward(gob, torch_bf16_to_bits(out), P, qb, kb, vb, scale)
    for t, ref in ((q.grad, dq), (k.grad, dk), (v.grad, dv)):
        compare(bf16_bits_to_f32(torch_bf16_to_bits(t)), ref)


@pytest.mark.parametrize("b,n,h,grp,dh", [(2, 520, 2, 2, 64), (1, 768, 1, 4, 128)])
def test_attention_default_positions_against_oracle(cuda, b, n, h, grp, dh):
    """Without positions (0..n-1) the products skip the masked tiles (UFP8_TILES_*): same results."""
    import torch
    from macrogpt_jax_b200.attention import softmax_attention
    rng = np.random.default_rng(n + grp)
    qb = bf16_normal(rng, (b, n, h * grp, dh))
    kb, vb = bf16_normal(rng, (b, n, h, dh)), bf16_normal(rng, (b, n, h, dh))
    seg = _segments(b, n, rng)
    q, k, v = (bits_to_torch_bf16(t, cuda).requires_grad_(True) for t in (qb, kb, vb))
    segt = torch.from_numpy(seg).to(cuda)
    out = softmax_attention(q, k, v, None, segt, None, segt, scale=dh ** -0.5)
    gob = bf16_normal(rng, (b, n, h * grp, dh))
    out.backward(bits_to_torch_bf16(gob, cuda))
    torch.cuda.synchronize()
    ro, P = oa.attention_forward(qb, kb, vb, seg, seg, None, None, dh ** -0.5)
    compare(bf16_bits_to_f32(torch_bf16_to_bits(out)), bf16_bits_to_f32(ro))
    dq, dk, dv = oa.attention_backward(gob, torch_bf16_to_bits(out), P, qb, kb, vb, dh ** -0.5)
    for t, ref in ((q.grad, dq), (k.grad, dk), (v.grad, dv)):
        compare(bf16_bits_to_f32(torch_bf16_to_bits(t)), ref)


def test_attention_segments_isolate(cuda):
    """Changing the keys of one document leaves the other documents' outputs bit-identical."""
    import torch
    from macrogpt_jax_b200.attention import softmax_attention
    rng = np.random.default_rng(11)
    b, n, h, dh = 1, 128, 2, 64
    q, k, v = (bits_to_torch_bf16(bf16_normal(rng, s), cuda) for s in ((b, n, h, dh), (b, n, h, dh), (b, n, h, dh)))
    seg = torch.zeros((b, n), dtype=torch.int32, device=cuda)
    seg[:, 64:] = 1
    a = softmax_attention(q, k, v, None, seg, None, seg, scale=0.125)
    k2 = k.clone()
    k2[:, 100] += 1
    a2 = softmax_attention(q, k2, v, None, seg, None, seg, scale=0.125)
    assert torch.equal(a[:, :64], a2[:, :64]) and not torch.equal(a[:, 64:], a2[:, 64:])


def test_transformer_layer_end_to_end(cuda):
    """SoftmaxAttention (FP8 projections, RoPE, softmax attention, GQA) inside TransformerLayer:
    forward and backward run, are finite and deterministic, and the attention half equals its
    pieces composed by hand (same kernels, same bits)."""
    import torch
    from macrogpt_jax_b200.attention import softmax_attention
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.layer import TransformerLayer
    from macrogpt_jax_b200.soft_attn import SoftmaxAttention
    d = 256
    init = Einsum.override(initializer=scaled_normal_init(d ** -0.5))
    attn = SoftmaxAttention.override(kq_d=64, kv_heads=2, kv_q_ratio=2, q=init, k=init, v=init, o=init)
    layer = TransformerLayer(d, attn=attn, rngs=Rngs(0))
    gen = torch.Generator(device=cuda)
    gen.manual_seed(2)
    x = torch.randn((2, 64, d), generator=gen, device=cuda).to(torch.bfloat16)
    seg = torch.zeros((2, 64), dtype=torch.int32, device=cuda)
    seg[1, 40:] = 1

    def run():
        xl = x.detach().requires_grad_(True)
        y = layer(xl, query_segment_ids=seg)
        y.float().square().mean().backward()
        return y.detach(), xl.grad.detach()

    y1, g1 = run()
    layer.zero_grad(set_to_none=True)
    y2, g2 = run()
    assert torch.isfinite(y1).all() and torch.isfinite(g1).all()
    assert torch.equal(y1, y2) and torch.equal(g1, g2)
    a = layer.attn
    xn = layer.attn_norm(x)
    q, k, v = a.project_qkv(xn)
    pos = torch.arange(64, device=cuda)
    q, k = a.rope(q, position_ids=pos), a.rope(k, position_ids=pos)
    o = softmax_attention(q.reshape(2, 64, 4, 64), k, v, pos, seg, pos, seg, scale=a.scale())
    assert torch.equal(a.project_out(o.reshape(2, 64, 2, 2, 64)), a(xn, query_segment_ids=seg))
