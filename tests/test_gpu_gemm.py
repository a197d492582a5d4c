"""tcgen05 FP8 GEMM vs the oracle: operand majors, formats, ragged tails, batching,
K concatenation, f32 output and the fused SwiGLU / dSwiGLU epilogues.

Operands are quantised by the oracle and uploaded as fp8 codes, so these tests check the
contraction independently of the quantize kernel."""
import numpy as np
import pytest

from oracle import fp8 as ofp8
from oracle import path as op

from helpers import bf16_bits_to_f64, compare, torch_bf16_to_bits, bits_to_torch_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(params=[1, 2, 3, 4, 5], ids=["single_cta", "cta_pair", "cta_pair_direct", "cta_pair_wide",
                                             "cta_pair_n512"], autouse=True)
def variant(request, cuda):
    """Runs every test with the one-CTA kernel and with the CTA-pair kernel, the latter with
    its staged epilogues (U / G of DSWIGLU through TMA), with the direct ones, with ring
    stages of two 128-byte K chunks, and with 256 x 512 tiles (bf16 STORE and SWIGLU)."""
    from macrogpt_jax_b200 import _capi
    _capi.set_gemm_variant(request.param)
    yield request.param
    _capi.set_gemm_variant(0)


def _upload(q: op.Q, cuda, transpose=False):
    import torch
    from macrogpt_jax_b200 import ops
    codes = q.codes
    if transpose:
        codes = np.ascontiguousarray(np.swapaxes(codes, -1, -2))
    t = torch.from_numpy(np.ascontiguousarray(codes)).to(cuda).view(ops.FP8_DTYPE[q.fmt])
    inv = torch.tensor([float(q.inv)], dtype=torch.float32, device=cuda)
    return ops.Fp8Tensor(t, inv, torch.tensor([float(q.amax)], dtype=torch.float32, device=cuda))


def _rand_q(rng, shape, fmt, std=1.0):
    return op.quant(op.bf16_normal(rng, shape, std), fmt)


@pytest.mark.parametrize("a_major", [0, 1])
@pytest.mark.parametrize("b_major", [0, 1])
@pytest.mark.parametrize("fmts", [(0, 0), (1, 0), (0, 1)])
def test_gemm_layouts(cuda, a_major, b_major, fmts):
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(100 + 10 * a_major + b_major)
    M, N, K = 384, 512, 640
    qa = _rand_q(rng, (M, K), fmts[0])
    qb = _rand_q(rng, (N, K), fmts[1])
    ta = _upload(qa, cuda, transpose=a_major == 1)
    tb = _upload(qb, cuda, transpose=b_major == 1)
    d = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ops.gemm(ops.operand(ta, a_major, K if a_major == 0 else M), ops.operand(tb, b_major, K if b_major == 0 else N),
             M, N, K, d, N)
    ref = op.gemm(qa, qb, "mk", "nk", "mn")
    compare(bf16_bits_to_f64(torch_bf16_to_bits(d)), bf16_bits_to_f64(ref))


@pytest.mark.parametrize("M,N,K", [(1, 16, 16), (130, 300, 48), (257, 129, 144), (128, 256, 128), (1000, 40, 1040),
                                   (384, 512, 256), (600, 700, 96)])
def test_gemm_ragged(cuda, M, N, K):
    """Tails in M, N and K (K-major operands; pitches padded to 16 bytes as TMA needs)."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(M * 7 + N)
    qa = _rand_q(rng, (M, K), 0)
    qb = _rand_q(rng, (N, K), 0)
    ta, tb = _upload(qa, cuda), _upload(qb, cuda)
    ldd = N + 3  # odd output pitch exercises the scalar store path
    dbuf = torch.full((M, ldd), float("nan"), dtype=torch.bfloat16, device=cuda)
    ops.gemm(ops.operand(ta, 0, K), ops.operand(tb, 0, K), M, N, K, dbuf, ldd)
    out = torch_bf16_to_bits(dbuf)
    ref = op.gemm(qa, qb, "mk", "nk", "mn")
    compare(bf16_bits_to_f64(out[:, :N]), bf16_bits_to_f64(ref))
    assert np.isnan(bf16_bits_to_f64(out[:, N:])).all(), "GEMM wrote outside [M, N]"


def test_gemm_f32_out_and_batch(cuda):
    """D[g] = A (broadcast) x B[g], fp32 output, MN-major operands (the dW shape)."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(5)
    G, M, N, K = 3, 256, 384, 512
    qa = _rand_q(rng, (M, K), 0)
    qb = _rand_q(rng, (G, N, K), 1)
    ta = _upload(qa, cuda, transpose=True)        # [K, M]
    tb = _upload(qb, cuda, transpose=True)        # [G, K, N]
    d = torch.empty((G, M, N), dtype=torch.float32, device=cuda)
    ops.gemm(ops.operand(ta, 1, M), ops.operand(tb, 1, N, K * N, G), M, N, K, d, N, M * N, batch=G)
    ref = op.gemm(qa, qb, "mk", "gnk", "gmn", out_f32=True)
    compare(d.cpu().numpy(), ref, rel_tol=1e-5, cos_tol=0.999999)


def test_gemm_k_batches(cuda):
    """D = sum_i A[i] B[i]^T (the dx contraction over [up, gate])."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(6)
    M, N, K = 256, 256, 384
    qa = _rand_q(rng, (2, M, K), 1)
    qb = _rand_q(rng, (2, N, K), 0)
    ta, tb = _upload(qa, cuda), _upload(qb, cuda)
    d = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ops.gemm(ops.operand(ta, 0, K, M * K, 2), ops.operand(tb, 0, K, N * K, 2), M, N, K, d, N, k_batches=2)
    ref = op.gemm(qa, qb, "imk", "ink", "mn")
    compare(bf16_bits_to_f64(torch_bf16_to_bits(d)), bf16_bits_to_f64(ref))


def test_gemm_k_zero(cuda):
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(8)
    qa = _rand_q(rng, (64, 16), 0)
    ta = _upload(qa, cuda)
    d = torch.full((64, 32), 1.0, dtype=torch.bfloat16, device=cuda)
    ops.gemm(ops.operand(ta, 0, 16), ops.operand(ta, 0, 16), 64, 32, 0, d, 32)
    assert (d == 0).all()


@pytest.mark.parametrize("T,d,h", [(256, 128, 256), (200, 256, 384), (512, 384, 640), (300, 128, 208)])
def test_swiglu_epilogue(cuda, T, d, h):
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(T + h)
    qx = _rand_q(rng, (T, d), 0)
    qw = op.quant(op.bf16_normal(rng, (2, d, h), d ** -0.5), 0)
    tx, tw = _upload(qx, cuda), _upload(qw, cuda)
    ug = torch.empty((2, T, h), dtype=torch.bfloat16, device=cuda)
    hid = torch.empty((T, h), dtype=torch.bfloat16, device=cuda)
    amax = torch.empty(1, dtype=torch.float32, device=cuda)
    ops.gemm(ops.operand(tx, 0, d), ops.operand(tw, 1, h, d * h, 2), T, h, d, ug, h, T * h,
             epilogue=ops.C.EPI_SWIGLU, h=hid, ldh=h, amax_out=amax)
    acc = np.einsum("td,idh->ith", qx.deq(), qw.deq())
    ref_ug = ofp8.f32_to_bf16_bits(acc.astype(np.float32) * op.alpha_of(qx, qw))
    ref_h = op.swiglu(ref_ug[0], ref_ug[1])
    got_ug, got_h = torch_bf16_to_bits(ug), torch_bf16_to_bits(hid)
    compare(bf16_bits_to_f64(got_ug), bf16_bits_to_f64(ref_ug))
    compare(bf16_bits_to_f64(got_h), bf16_bits_to_f64(ref_h))
    # H computed from the GPU's own U, G must match to within one bf16 rounding step.
    h_from_gpu = bf16_bits_to_f64(op.swiglu(got_ug[0], got_ug[1]))
    assert np.abs(bf16_bits_to_f64(got_h) - h_from_gpu).max() <= 2 ** -7 * np.abs(h_from_gpu).max()
    assert amax.item() == float(ofp8.amax_bits(got_h))


@pytest.mark.parametrize("T,d,h", [(256, 128, 256), (200, 256, 384), (520, 256, 464)])
def test_dswiglu_epilogue(cuda, T, d, h):
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(T * 3 + h)
    qdy = _rand_q(rng, (T, d), 1, 1e-3)
    qwd = op.quant(op.bf16_normal(rng, (h, d), h ** -0.5), 0)
    ug_bits = op.bf16_normal(rng, (2, T, h))
    tdy, twd = _upload(qdy, cuda), _upload(qwd, cuda)
    ug = bits_to_torch_bf16(ug_bits, cuda)
    dug = torch.empty((2, T, h), dtype=torch.bfloat16, device=cuda)
    amax = torch.empty(1, dtype=torch.float32, device=cuda)
    ops.gemm(ops.operand(tdy, 0, d), ops.operand(twd, 0, d), T, h, d, dug, h, T * h,
             epilogue=ops.C.EPI_DSWIGLU, ug=ug, ldug=h, ug_batch_stride=T * h, amax_out=amax)
    dh = np.einsum("td,hd->th", qdy.deq(), qwd.deq()).astype(np.float32) * op.alpha_of(qdy, qwd)
    du, dg = op.dswiglu(dh, ug_bits[0], ug_bits[1])
    got = torch_bf16_to_bits(dug)
    compare(bf16_bits_to_f64(got[0]), bf16_bits_to_f64(du))
    compare(bf16_bits_to_f64(got[1]), bf16_bits_to_f64(dg))
    assert amax.item() == float(ofp8.amax_bits(got))


def test_many_tiles(cuda):
    """More tiles than resident CTAs / clusters (several persistent passes, both TMEM buffers)."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(9)
    M, N, K = 4096, 2560, 256
    qa = _rand_q(rng, (M, K), 0)
    qb = _rand_q(rng, (N, K), 0)
    ta, tb = _upload(qa, cuda), _upload(qb, cuda)
    d = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    ops.gemm(ops.operand(ta, 0, K), ops.operand(tb, 0, K), M, N, K, d, N)
    ref = op.gemm(qa, qb, "mk", "nk", "mn")
    compare(bf16_bits_to_f64(torch_bf16_to_bits(d)), bf16_bits_to_f64(ref))


def test_device_status_clean(cuda):
    from macrogpt_jax_b200 import ops
    assert ops.device_status() == 0
