"""Next-token cross-entropy on a B200: the ufp8_xent_* kernels and the XENT GEMM epilogue against
the oracle (oracle/xent.py), and the fused OutputHead loss against the oracle's head and against
the generic (chunked, unfused) path.

Tolerances.  The loss is f32 arithmetic on bf16 logits: lse within 2e-6 relative of the oracle's
float64 logsumexp.  exp is the MUFU approximation on the GPU and numpy's f32 exp in the oracle's
gradient, so a gradient element that sits on a rounding boundary of its output format may round
the other way: at most 1 % of the bf16 gradients and 0.2 % of the fp8 codes may differ, and only
by one step.  Module-level results go through FP8 GEMMs and use the GEMM tolerance of helpers.py."""
import numpy as np
import pytest

from oracle import fp8 as ofp8
from oracle import path as op
from oracle import xent as ox

from helpers import bf16_bits_to_f64, bits_to_torch_bf16, compare, torch_bf16_to_bits, torch_fp8_to_codes

pytestmark = pytest.mark.gpu



def _labels(rng, T, V, oob=True):
    lab = rng.integers(-V, V, T).astype(np.int32)
    if oob and T >= 4:
        lab[1], lab[3] = V, -V - 1  # no column: NaN loss
    return lab


def _np(t):
    return t.detach().cpu().numpy()


def _dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


@pytest.mark.parametrize("T,V,pad", [(0, 10, 0), (1, 1, 0), (5, 7, 3), (64, 1000, 0), (33, 8200, 8),
                                     (17, 300, 1), (8, 128256, 0)])
def test_xent_rows_against_oracle(cuda, T, V, pad):
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(T * 31 + V)
    lb = op.bf16_normal(rng, (T, V + pad), 3.0)
    labels = _labels(rng, T, V)
    mask = rng.integers(0, 2, T).astype(np.uint8)
    logits = bits_to_torch_bf16(lb, cuda)
    lse, loss, qrow = ops.xent_rows(logits, _dev(labels, cuda), _dev(mask, cuda), V)
    rl, rloss, rq = ox.xent_rows(lb[:, :V], labels, mask)
    lse, loss, qrow = _np(lse), _np(loss), _np(qrow)
    np.testing.assert_allclose(lse, rl, rtol=2e-6, atol=1e-6)
    assert np.array_equal(np.isnan(loss), np.isnan(rloss))
    ok = ~np.isnan(rloss)
    np.testing.assert_allclose(loss[ok], rloss[ok], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(qrow, rq, atol=2e-6)


def _quantised_head(cuda, rng, T, d, V, std=3.0):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    xb = op.bf16_normal(rng, (T, d))
    wb = op.bf16_normal(rng, (d, V), std * d ** -0.5)
    qx = ops.quantize(bits_to_torch_bf16(xb, cuda), C.E4M3)
    qw = ops.quantize_head_weight(bits_to_torch_bf16(wb, cuda))
    # the same contraction with the plain STORE epilogue
    Vp = qw.q.shape[1]
    plain = torch.empty((T, Vp), dtype=torch.bfloat16, device=cuda)
    ops.gemm(ops.operand(qx, C.K_MAJOR, d), ops.operand(qw, C.MN_MAJOR, Vp), T, V, d, plain, Vp)
    return qx, qw, plain


@pytest.mark.parametrize("T,d,V,cap", [(256, 256, 1024, 0.0), (300, 128, 1000, 0.0), (300, 128, 1000, 15.0),
                                       (1, 256, 4112, 0.0), (512, 512, 8192, 15.0)])
def test_xent_gemm_epilogue(cuda, T, d, V, cap):
    """The XENT epilogue stores the STORE epilogue's logits (soft-capped as the oracle caps them) and
    per-128-column partials that match the stored logits; ufp8_xent_combine then equals
    ufp8_xent_forward on the same logits."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(T + d + V)
    qx, qw, plain = _quantised_head(cuda, rng, T, d, V)
    logits, stats = ops.head_logits(qx, qw, V, cap)
    torch.cuda.synchronize()
    got = torch_bf16_to_bits(logits[:, :V])
    ref = torch_bf16_to_bits(plain[:, :V])
    if cap:
        ref = ox.soft_cap(ref, cap)
        diff = got != ref
        assert diff.mean() <= 1e-3, f"{diff.mean():.2e} of the capped logits differ"
        assert (np.abs(bf16_bits_to_f64(got[diff]) - bf16_bits_to_f64(ref[diff])) <=
                np.abs(bf16_bits_to_f64(ref[diff])) * 2 ** -7).all()
    else:
        assert np.array_equal(got, ref)
    c = bf16_bits_to_f64(got)
    groups = (V + 127) // 128
    st = _np(stats).astype(np.float64)
    for j in range(groups):
        blk = c[:, 128 * j: min(128 * j + 128, V)]
        m = blk.max(axis=1)
        s = np.exp(blk - m[:, None]).sum(axis=1)
        assert np.array_equal(st[:, j, 0], m)
        np.testing.assert_allclose(st[:, j, 1], s, rtol=1e-5)
    labels = _labels(rng, T, V)
    mask = rng.integers(0, 2, T).astype(np.uint8)
    lab_t, mask_t = _dev(labels, cuda), _dev(mask, cuda)
    a = ops.xent_combine(stats, logits, V, lab_t, mask_t)
    b = ops.xent_rows(logits, lab_t, mask_t, V)
    rl, rloss, rq = ox.xent_rows(got, labels, mask)
    for x, y in zip(a, b):
        x, y = _np(x), _np(y)
        assert np.array_equal(np.isnan(x), np.isnan(y))
        ok = ~np.isnan(x)
        np.testing.assert_allclose(x[ok], y[ok], rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(_np(a[0]), rl, rtol=2e-6, atol=1e-6)


@pytest.mark.parametrize("T,V,pad,cap,fmt", [(64, 1000, 0, 0.0, 2), (33, 8200, 8, 15.0, 2), (5, 7, 3, 0.0, 2),
                                             (64, 1000, 0, 0.0, 1), (40, 8200, 8, 0.0, 0), (33, 4096, 0, 15.0, 1),
                                             (5, 7, 3, 0.0, 1), (0, 16, 0, 0.0, 1), (4, 128256, 0, 0.0, 1)])
def test_xent_backward_against_oracle(cuda, T, V, pad, cap, fmt):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(T * 7 + V + fmt)
    lb = op.bf16_normal(rng, (T, V + pad), 3.0)
    if cap:
        lb = ox.soft_cap(lb, cap)
    labels = _labels(rng, T, V, oob=(fmt == C.BF16))
    mask = rng.integers(0, 2, T).astype(np.uint8)
    dloss = rng.standard_normal(T).astype(np.float32)
    logits = bits_to_torch_bf16(lb, cuda)
    lab_t, mask_t = _dev(labels, cuda), _dev(mask, cuda)
    lse, _, qrow = ops.xent_rows(logits, lab_t, mask_t, V)
    out = ops.xent_grad(logits, lab_t, mask_t, lse, qrow, _dev(dloss, cuda), cap, fmt, V)
    torch.cuda.synchronize()
    if fmt == C.BF16:
        got = torch_bf16_to_bits(out)
        ref = ox.xent_backward(lb[:, :V], labels, mask, _np(lse), _np(qrow), dloss, cap, ox.BF16)
        diff = got != ref
        assert diff.mean() <= 1e-2 if diff.size else True
        step = np.abs(got[diff].astype(np.int32) - ref[diff].astype(np.int32))
        assert (step <= 1).all(), "a bf16 gradient differs by more than one step"
        return
    codes = torch_fp8_to_codes(out.q)[:, :V]
    ref, ramax, rinv = ox.xent_backward(lb[:, :V], labels, mask, _np(lse), _np(qrow), dloss, cap, fmt)
    assert _np(out.amax).view(np.uint32)[0] == np.array([ramax], np.float32).view(np.uint32)[0]
    assert _np(out.inv_scale).view(np.uint32)[0] == np.array([rinv], np.float32).view(np.uint32)[0]
    if T == 0:
        return
    diff = codes != ref
    assert diff.mean() <= 2e-3, f"{diff.mean():.2e} of the fp8 codes differ"
    assert ((codes[diff] & 0x80) == (ref[diff] & 0x80)).all()
    assert (np.abs((codes[diff] & 0x7F).astype(np.int32) - (ref[diff] & 0x7F).astype(np.int32)) <= 1).all()
    deq = ofp8.fp8_to_f64(codes, fmt)
    assert np.isfinite(deq).all()
    if not cap and ramax > 0:
        # the scale comes from the label column, which holds each row's largest |dl|
        assert np.abs(deq).max() == ofp8.FMAX[fmt]


def _head(cuda, d, V, cap, seed=0):
    import torch
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.head import OutputHead
    head = OutputHead.override(lm_head=Einsum.override(initializer=scaled_normal_init(3 * d ** -0.5)))(
        d, V, head_cap=cap, rngs=Rngs(seed))
    rng = np.random.default_rng(seed + 11)
    with torch.no_grad():
        head.norm.scale.copy_(bits_to_torch_bf16(op.bf16_normal(rng, (d,), 0.3), cuda) + 1)
    return head


@pytest.mark.parametrize("cap,V", [(None, 1000), ("tanh", 1000), ("tanh", 2048)])
def test_output_head_fused_loss_against_oracle(cuda, cap, V):
    """chunked_softmax_cross_entropy(inputs, activations, head.get_logits) takes the fused node; its
    loss and the gradients of the activations, the lm_head weight and the norm scale match the
    oracle's head (norm -> FP8 lm_head -> cap -> loss and its backward)."""
    import torch
    from macrogpt_jax_b200 import next_token_loss as ntl
    B, S, d = 2, 96, 256
    head = _head(cuda, d, V, cap)
    assert ntl._fused_head(head.get_logits) is head
    rng = np.random.default_rng(5)
    inputs = rng.integers(0, V, (B, S))
    xb = op.bf16_normal(rng, (B * S, d))
    x = bits_to_torch_bf16(xb, cuda).reshape(B, S, d).requires_grad_(True)
    loss = ntl.chunked_softmax_cross_entropy(_dev(inputs, cuda), x, head.get_logits, pad_token_id=0)
    loss.sum().backward()
    torch.cuda.synchronize()
    targets, mask = ox.ntp_args(inputs, pad_token_id=0)
    capv = 15.0 if cap else 0.0
    sb = torch_bf16_to_bits(head.norm.scale)
    wb = torch_bf16_to_bits(head.lm_head.w)
    rloss, sv = ox.head_forward(xb, sb, False, head.norm.eps, wb, targets.reshape(-1), mask.reshape(-1), capv)
    got = _np(loss).reshape(-1)
    np.testing.assert_allclose(got, rloss, atol=2e-2)
    assert np.abs(got - rloss).mean() <= 3e-3
    g = ox.head_backward(np.ones(B * S, np.float32), sv, xb, sb, False, targets.reshape(-1), mask.reshape(-1), capv)
    compare(bf16_bits_to_f64(torch_bf16_to_bits(x.grad)).reshape(-1), g["dx"].reshape(-1))
    compare(bf16_bits_to_f64(torch_bf16_to_bits(head.lm_head.w.grad)), bf16_bits_to_f64(g["dw"]))
    compare(_np(head.norm.scale.grad.float()), g["dscale"])


def test_fused_and_generic_paths_agree(cuda):
    """The generic path (any projection: the reference's chunking, checkpointed chunks, the
    bf16-logit kernels) against the fused node on the same head, and, with several chunks,
    against the oracle's head applied chunk by chunk.

    One chunk: the losses agree within the bf16 resolution of the logits (torch's soft cap divides
    by 15 through a reciprocal, the fused epilogue with an IEEE division, so a capped logit may
    differ by one bf16 step).  The gradients are two fp8 quantisations of the logit gradient with
    different scales (the generic Einsum takes max |dl| of the bf16 gradient, the fused node its
    bound from the row results): each term of dX = dL W^T may round by up to 2^-3 in either, so an
    element may differ by up to 2 x 2^-3 of its largest terms (max relative error 0.25); the cosine
    is the tight check.  Several chunks: every chunk quantises its input with its own scale, as the
    reference's chunks do, so the losses follow the per-chunk oracle, and the gradients differ from
    the fused node's by the input's e4m3 rounding as well (cosine 0.99)."""
    import torch
    from macrogpt_jax_b200 import next_token_loss as ntl
    B, S, d, V = 2, 96, 256, 1024
    head = _head(cuda, d, V, "tanh", seed=3)
    rng = np.random.default_rng(9)
    tokens = rng.integers(0, V, (B, S))
    inputs = _dev(tokens, cuda)
    xb = op.bf16_normal(rng, (B * S, d))

    def run(proj, chunk):
        x = bits_to_torch_bf16(xb, cuda).reshape(B, S, d).requires_grad_(True)
        head.zero_grad(set_to_none=True)
        loss = ntl.chunked_softmax_cross_entropy(inputs, x, proj, chunk_size=chunk)
        loss.sum().backward()
        return _np(loss), x.grad.float().cpu().numpy(), head.lm_head.w.grad.float().cpu().numpy()

    fused = run(head.get_logits, 1024)
    one = run(lambda a: head.get_logits(a), 1024)
    np.testing.assert_allclose(one[0], fused[0], atol=2e-2)
    assert np.abs(one[0] - fused[0]).mean() <= 2e-3
    compare(one[1], fused[1], rel_tol=0.25, cos_tol=0.998)
    compare(one[2], fused[2], rel_tol=0.25, cos_tol=0.998)
    chunked = run(lambda a: head.get_logits(a), 64)  # chunks of 64 and 32 positions
    targets, mask = ox.ntp_args(tokens)
    xs = xb.reshape(B, S, d)
    sb, wb = torch_bf16_to_bits(head.norm.scale), torch_bf16_to_bits(head.lm_head.w)
    for s0, e0 in ((0, 64), (64, 96)):
        rl, _ = ox.head_forward(xs[:, s0:e0].reshape(-1, d), sb, False, head.norm.eps, wb,
                                targets[:, s0:e0].reshape(-1), mask[:, s0:e0].reshape(-1), 15.0)
        got = chunked[0][:, s0:e0].reshape(-1)
        np.testing.assert_allclose(got, rl, atol=2e-2)
        assert np.abs(got - rl).mean() <= 3e-3
    compare(chunked[1], fused[1], rel_tol=0.25, cos_tol=0.99)
    compare(chunked[2], fused[2], rel_tol=0.25, cos_tol=0.99)


def test_full_vocabulary_properties(cuda):
    """Llama-3 vocabulary (128256 classes, d 4096) on 1024 tokens: the fused loss equals the
    logsumexp of the stored logits minus the label logit, and each row of the bf16 gradient of
    sum(loss) sums to zero (softmax sums to one)."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    T, d, V = 1024, 4096, 128256
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1)
    x = torch.randn((T, d), generator=gen, device=cuda).to(torch.bfloat16)
    w = (torch.randn((d, V), generator=gen, device=cuda) * d ** -0.5).to(torch.bfloat16)
    qx = ops.quantize(x, C.E4M3)
    qw = ops.quantize_head_weight(w)
    del w
    logits, stats = ops.head_logits(qx, qw, V, 15.0)
    labels = torch.randint(0, V, (T,), generator=gen, device=cuda, dtype=torch.int32)
    lse, loss, qrow = ops.xent_combine(stats, logits, V, labels, None)
    lf = logits[:, :V].float()
    ref_lse = torch.logsumexp(lf, dim=1)
    torch.testing.assert_close(lse, ref_lse, rtol=2e-6, atol=3e-5)
    torch.testing.assert_close(loss, ref_lse - lf.gather(1, labels.long()[:, None])[:, 0], rtol=2e-6, atol=5e-5)
    g0 = ops.xent_grad(logits, labels, None, lse, qrow, None, 0.0, C.BF16, V)
    rowsum = g0.float().sum(dim=1)  # sum_j softmax_j - 1, each term rounded to bf16
    assert rowsum.abs().max().item() < 5e-3
    g = ops.xent_grad(logits, labels, None, lse, qrow, None, 15.0, C.BF16, V).float()
    q = ops.xent_grad(logits, labels, None, lse, qrow, None, 15.0, C.E5M2, V)
    deq = q.q[:, :V].float() * q.inv_scale
    assert torch.isfinite(deq).all()
    assert ((deq - g).abs() <= 0.13 * g.abs() + 1e-5 * q.amax).all()
