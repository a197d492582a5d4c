"""The bf16 GEMM (tcgen05 kind::f16) with its STORE and AXPBY epilogues against float64 products
of the same bf16 operands, and Muon's Newton-Schulz orthogonalisation (ufp8_newton_schulz,
macrogpt_jax_b200.muon.orthogonalize) against the oracle (oracle/muon.py).

Bars: bf16 outputs max|D - R| <= 1e-2 max|R| and cosine >= 0.99999 (bf16 rounding of D, fp32
accumulation); f32 outputs 1e-4 and 0.999999.  Newton-Schulz: the GPU and the oracle's bf16
storage points differ first by the order of the fp32 accumulations, which moves an occasional
bf16 rounding of X, A or B by one step; each iteration then amplifies such differences along the
small singular directions (the polynomials' slope near 0 is 3.4 for 'muon' and up to 8.3 for the
first 'optimal' step), so after five steps an element may be off by a few per cent of the
largest: max|D - R| <= 0.1 max|R| with cosine >= 0.999 against the storage-point oracle, and
cosine >= 0.99 against the float64 algorithm (five steps of bf16 storage)."""
import numpy as np
import pytest

from oracle import muon as om
from oracle import path as op

from helpers import bf16_bits_to_f64, bits_to_torch_bf16, compare

pytestmark = pytest.mark.gpu


def _cmp(out, ref, f32):
    compare(out, ref, rel_tol=1e-4 if f32 else 1e-2, cos_tol=0.999999 if f32 else 0.99999)


@pytest.mark.parametrize("M,N,K,batch", [(256, 256, 128, 1), (264, 520, 136, 1), (128, 1000, 4096, 1),
                                         (512, 384, 200, 3)])
@pytest.mark.parametrize("am,bm", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("f32", [False, True])
def test_bf16_gemm_against_f64(cuda, M, N, K, batch, am, bm, f32):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(M + N + K + batch + 2 * am + bm)
    a_bits = op.bf16_normal(rng, (batch, M, K))
    b_bits = op.bf16_normal(rng, (batch, N, K))
    a_st = a_bits if am == C.K_MAJOR else np.ascontiguousarray(np.swapaxes(a_bits, 1, 2))
    b_st = b_bits if bm == C.K_MAJOR else np.ascontiguousarray(np.swapaxes(b_bits, 1, 2))
    at, bt = bits_to_torch_bf16(a_st, cuda), bits_to_torch_bf16(b_st, cuda)
    d = torch.empty((batch, M, N), dtype=torch.float32 if f32 else torch.bfloat16, device=cuda)
    ops.gemm(ops.bf16_operand(at, am, K if am == C.K_MAJOR else M, M * K, batch),
             ops.bf16_operand(bt, bm, K if bm == C.K_MAJOR else N, N * K, batch),
             M, N, K, d, N, M * N, batch=batch)
    torch.cuda.synchronize()
    ref = np.einsum("bmk,bnk->bmn", bf16_bits_to_f64(a_bits), bf16_bits_to_f64(b_bits))
    _cmp(d.double().cpu().numpy(), ref, f32)


@pytest.mark.parametrize("am,bm", [(0, 0), (0, 1), (1, 0)])
@pytest.mark.parametrize("f32", [False, True])
def test_bf16_gemm_axpby(cuda, am, bm, f32):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    M, N, K, batch, alpha, beta = 264, 392, 520, 2, 0.75, -1.25
    rng = np.random.default_rng(7 + am + bm)
    a_bits = op.bf16_normal(rng, (batch, M, K))
    b_bits = op.bf16_normal(rng, (batch, N, K))
    c_bits = op.bf16_normal(rng, (batch, M, N), 8.0)
    a_st = a_bits if am == C.K_MAJOR else np.ascontiguousarray(np.swapaxes(a_bits, 1, 2))
    b_st = b_bits if bm == C.K_MAJOR else np.ascontiguousarray(np.swapaxes(b_bits, 1, 2))
    ct = bits_to_torch_bf16(c_bits, cuda)
    at, bt = bits_to_torch_bf16(a_st, cuda), bits_to_torch_bf16(b_st, cuda)  # alive until the GEMM ran
    d = torch.empty((batch, M, N), dtype=torch.float32 if f32 else torch.bfloat16, device=cuda)
    ops.gemm(ops.bf16_operand(at, am, K if am == C.K_MAJOR else M, M * K, batch),
             ops.bf16_operand(bt, bm, K if bm == C.K_MAJOR else N, N * K, batch),
             M, N, K, d, N, M * N, batch=batch, epilogue=C.EPI_AXPBY, axpby=(ct, N, M * N, alpha, beta))
    torch.cuda.synchronize()
    ref = alpha * np.einsum("bmk,bnk->bmn", bf16_bits_to_f64(a_bits), bf16_bits_to_f64(b_bits)) + \
        beta * bf16_bits_to_f64(c_bits)
    _cmp(d.double().cpu().numpy(), ref, f32)


def test_bf16_gemm_rejects_mixed_and_fp8_epilogues(cuda):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    a = torch.zeros((64, 64), dtype=torch.bfloat16, device=cuda)
    q = ops.quantize(a, C.E4M3)
    d = torch.empty((64, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(C.UFP8Error, match="both be fp8 or both be bf16"):
        ops.gemm(ops.bf16_operand(a, C.K_MAJOR, 64), ops.operand(q, C.K_MAJOR, 64), 64, 64, 64, d, 64)
    with pytest.raises(C.UFP8Error, match="STORE, AXPBY and ATTN"):
        ops.gemm(ops.bf16_operand(a, C.K_MAJOR, 64), ops.bf16_operand(a, C.K_MAJOR, 64), 64, 64, 64, d, 64,
                 epilogue=C.EPI_SWIGLU, h=d, ldh=64, amax_out=torch.empty(1, device=cuda))


@pytest.mark.parametrize("shape", [(1, 256, 512), (1, 512, 256), (3, 384, 384), (2, 128, 1024), (1, 1200, 600)])
@pytest.mark.parametrize("method", ["muon", "optimal"])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_orthogonalize_against_oracle(cuda, shape, method, dtype):
    import torch
    from macrogpt_jax_b200 import muon
    rng = np.random.default_rng(sum(shape) + len(method))
    g = rng.standard_normal(shape).astype(np.float32) * 0.02
    tdt = torch.float32 if dtype == "f32" else torch.bfloat16
    gt = torch.from_numpy(g).to(cuda).to(tdt)
    g_in = gt.float().cpu().numpy()  # the values the kernel reads (bf16-rounded for bf16 input)
    out = muon.orthogonalize(gt, method=method)
    torch.cuda.synchronize()
    assert out.shape == gt.shape and out.dtype == tdt
    co = om.coefficients(5, method)
    ref = om.orthogonalize_bf16(g_in, co, out_f32=dtype == "f32")
    got = out.float().cpu().numpy()
    compare(got, ref, rel_tol=0.1, cos_tol=0.999)
    r64 = om.orthogonalize_f64(g_in, co)
    cos = float((got.astype(np.float64) * r64).sum() / (np.linalg.norm(got) * np.linalg.norm(r64)))
    assert cos > 0.99


def test_orthogonalize_shapes_determinism_and_errors(cuda):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import muon
    gen = torch.Generator(device=cuda)
    gen.manual_seed(3)
    g4 = torch.randn((2, 3, 128, 256), generator=gen, device=cuda)
    a = muon.orthogonalize(g4)
    b = muon.orthogonalize(g4)
    assert a.shape == g4.shape and torch.equal(a, b)  # bit-identical runs
    flat = muon.orthogonalize(g4.reshape(6, 128, 256)).reshape(g4.shape)
    assert torch.equal(a, flat)
    one = muon.orthogonalize(g4[1, 2])
    assert torch.equal(one, a[1, 2])  # slices are independent
    with pytest.raises(ValueError):
        muon.orthogonalize(torch.zeros(8, device=cuda))
    with pytest.raises(C.UFP8Error, match="multiples of 8"):
        muon.orthogonalize(torch.zeros((12, 64), device=cuda))


@pytest.mark.parametrize("mask", [1, 2, 3])
def test_bf16_gemm_tile_masks(cuda, mask):
    """UFP8_TILES_LOWER computes exactly the 256 x 256 tiles on or below the diagonal (D elsewhere
    untouched); K_TO_DIAG / K_FROM_DIAG contract M tile m over K < 256 (m + 1) / K >= 256 m of each
    K slice (k_batches 2 here)."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    M, N, K, kb = 640, 768 if mask == 1 else 128, 640, 1 if mask == 1 else 2
    rng = np.random.default_rng(40 + mask)
    a_bits = op.bf16_normal(rng, (kb, M, K))
    b_bits = op.bf16_normal(rng, (kb, N, K))
    at, bt = bits_to_torch_bf16(a_bits, cuda), bits_to_torch_bf16(b_bits, cuda)
    d = torch.full((M, N), -7.0, dtype=torch.float32, device=cuda)
    desc_kw = dict(k_batches=kb) if kb > 1 else {}
    ops.gemm(ops.bf16_operand(at, C.K_MAJOR, K, M * K, kb), ops.bf16_operand(bt, C.K_MAJOR, K, N * K, kb),
             M, N, K, d, N, tile_mask=mask, **desc_kw)
    torch.cuda.synchronize()
    a64, b64 = bf16_bits_to_f64(a_bits), bf16_bits_to_f64(b_bits)
    ref = np.full((M, N), -7.0)
    for mt in range((M + 255) // 256):
        rows = slice(256 * mt, min(256 * mt + 256, M))
        if mask == 1:
            cols = slice(0, min(256 * mt + 256, N))
            ref[rows, cols] = np.einsum("mk,nk->mn", a64[0, rows], b64[0, cols])
        else:
            ks = slice(0, 256 * (mt + 1)) if mask == 2 else slice(256 * mt, K)
            ref[rows] = sum(a64[s, rows, ks] @ b64[s, :, ks].T for s in range(kb))
    got = d.double().cpu().numpy()
    np.testing.assert_array_equal(got == -7.0, ref == -7.0)
    _cmp(got, ref, True)


@pytest.mark.parametrize("b_major", [0, 1])
def test_bf16_gemm_batch_group(cuda, b_major):
    """batch_group 3: product g (of 6) reads B slice g / 3 (the key / value head shared by a group
    of query heads), slices laid out with a pitch smaller than the row pitch as the attention's
    [token, head, d] tensors are."""
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    import torch
    G, grp, M, N, K = 6, 3, 320, 128, 192
    rng = np.random.default_rng(50 + b_major)
    a_bits = op.bf16_normal(rng, (G, M, K))
    if b_major == C.K_MAJOR:
        b_bits = op.bf16_normal(rng, (N, G // grp, K))  # [n, head, k]: slice pitch K, row pitch heads * K
        bt = bits_to_torch_bf16(b_bits, cuda)
        bop = ops.bf16_operand(bt, C.K_MAJOR, (G // grp) * K, K, G // grp, grp)
        bmat = lambda s: b_bits[:, s, :]  # noqa: E731  [N, K]
    else:
        b_bits = op.bf16_normal(rng, (K, G // grp, N))  # [k, head, n]: MN-major
        bt = bits_to_torch_bf16(b_bits, cuda)
        bop = ops.bf16_operand(bt, C.MN_MAJOR, (G // grp) * N, N, G // grp, grp)
        bmat = lambda s: b_bits[:, s, :].T  # noqa: E731
    at = bits_to_torch_bf16(a_bits, cuda)
    d = torch.empty((G, M, N), dtype=torch.float32, device=cuda)
    ops.gemm(ops.bf16_operand(at, C.K_MAJOR, K, M * K, G), bop, M, N, K, d, N, M * N, batch=G)
    torch.cuda.synchronize()
    a64 = bf16_bits_to_f64(a_bits)
    ref = np.stack([a64[g] @ bf16_bits_to_f64(np.ascontiguousarray(bmat(g // grp))).T for g in range(G)])
    _cmp(d.double().cpu().numpy(), ref, True)
