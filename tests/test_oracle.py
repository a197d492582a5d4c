"""The oracle itself, on the CPU: its fp8 casts pinned against ml_dtypes 0.5.4 (the
reference's cast library), its contractions against an independent einsum (torch), its
gating derivative against autograd, and the committed golden fixtures."""
from pathlib import Path

import ml_dtypes
import numpy as np
import pytest
import torch

from oracle import fp8, path

GOLDEN = Path(__file__).resolve().parent / "golden" / "golden_v1.npz"
ALL_BF16 = np.arange(65536, dtype=np.uint32).astype(np.uint16)


@pytest.mark.parametrize("fmt,dt", [(fp8.E4M3, ml_dtypes.float8_e4m3fn), (fp8.E5M2, ml_dtypes.float8_e5m2)])
@pytest.mark.parametrize("scale", [1.0, 448 / 3.0, 1e-3, 7.123, 1e30, 2.0 ** -20, 57344.0])
def test_cast_matches_ml_dtypes_on_every_bf16(fmt, dt, scale):
    """Round to nearest even, subnormals, overflow (NaN for e4m3fn, inf for e5m2)."""
    with np.errstate(all="ignore"):
        p = fp8.bf16_bits_to_f32(ALL_BF16) * np.float32(scale)
        ref = p.astype(dt).view(np.uint8)
    mine = fp8.f32_to_fp8(p, fmt)
    nan = np.isnan(p)
    assert (mine[~nan] == ref[~nan]).all()
    assert (mine[nan] == (0x7F if fmt == fp8.E4M3 else 0x7E)).all()


@pytest.mark.parametrize("fmt", [fp8.E4M3, fp8.E5M2])
def test_fast_cast_equals_restatement(fmt):
    rng = np.random.default_rng(1)
    p = np.concatenate([rng.standard_normal(200_000).astype(np.float32) * np.float32(300),
                        fp8.bf16_bits_to_f32(ALL_BF16)])
    with np.errstate(all="ignore"):
        assert (fp8.f32_to_fp8_fast(p, fmt) == fp8.f32_to_fp8(p, fmt)).all()


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(2)
    v = np.concatenate([rng.standard_normal(100_000).astype(np.float32) * np.float32(1e3),
                        rng.integers(0, 2 ** 32, 100_000, dtype=np.uint64).astype(np.uint32).view(np.float32),
                        np.array([np.inf, -np.inf, 3.4e38, -3.4e38, 1e-45, 0.0, -0.0], np.float32)])
    mine = fp8.f32_to_bf16_bits(v)
    ref = torch.from_numpy(v).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    nan = np.isnan(v)
    assert (mine[~nan] == ref[~nan]).all()
    assert np.isnan(fp8.bf16_bits_to_f32(mine[nan])).all()


def test_decode_table_matches_ml_dtypes():
    for fmt, dt in ((fp8.E4M3, ml_dtypes.float8_e4m3fn), (fp8.E5M2, ml_dtypes.float8_e5m2)):
        codes = np.arange(256, dtype=np.uint8)
        ref = codes.view(dt).astype(np.float64)
        mine = fp8.fp8_to_f64(codes, fmt)
        assert np.array_equal(np.isnan(mine), np.isnan(ref))
        assert (mine[~np.isnan(mine)] == ref[~np.isnan(ref)]).all()


def test_quantize_recipe_edges():
    # amax == 0 -> scale 1, inverse scale 1
    q, a, inv = fp8.quantize_bits(np.zeros(10, np.uint16), fp8.E4M3)
    assert a == 0 and inv == 1 and (q == 0).all()
    # empty tensor
    q, a, inv = fp8.quantize_bits(np.zeros(0, np.uint16), fp8.E5M2)
    assert q.size == 0 and a == 0 and inv == 1
    # the tensor's own max maps to FMAX exactly
    x = fp8.f32_to_bf16_bits(np.array([0.5, -3.0, 1.25], np.float32))
    q, a, inv = fp8.quantize_bits(x, fp8.E4M3)
    assert a == np.float32(3.0) and q[1] == 0xFE  # -448
    # denormal amax: FMAX/amax overflows, s is capped at FLT_MAX, so the products stay finite:
    # x = 2^-133 (bf16 0x0001): 2^-133 * FLT_MAX = 2^-6 * (2 - 2^-23) rounds to 2^-5 in both
    # formats, 0 stays 0, and code * inv_scale (2^-128) gives x back exactly
    x = np.array([0x0001, 0x0000, 0x8001], np.uint16)
    q, a, inv = fp8.quantize_bits(x, fp8.E4M3)
    assert inv == np.float32(2.0 ** -128) and list(q) == [0x10, 0x00, 0x90]
    q, _, _ = fp8.quantize_bits(x, fp8.E5M2)
    assert list(q) == [0x28, 0x00, 0xA8]
    # amax around 1e-37 (normal bf16): no NaN, dequantised values close to x
    for fmt in (fp8.E4M3, fp8.E5M2):
        xb = fp8.f32_to_bf16_bits(np.array([1e-37, -3e-38, 5e-38, 0.0], np.float32))
        q, a, inv = fp8.quantize_bits(xb, fmt)
        deq = fp8.fp8_to_f64(q, fmt) * np.float64(inv)
        ref = fp8.bf16_bits_to_f32(xb).astype(np.float64)
        assert np.isfinite(deq).all()
        assert np.abs(deq - ref).max() <= 0.13 * np.abs(ref).max()
    # a NaN element makes amax NaN and every code NaN
    x = fp8.f32_to_bf16_bits(np.array([1.0, np.nan], np.float32))
    q, a, inv = fp8.quantize_bits(x, fp8.E4M3)
    assert np.isnan(a) and (q == 0x7F).all()


@pytest.mark.parametrize("expr,xs,ws", [
    ("bnd,idh->ibnh", (2, 3, 32), (2, 32, 48)),       # GMLP fused gate/up (ueaj/model/mlp.py:79)
    ("bnh,hd->bnd", (2, 3, 48), (48, 32)),            # GMLP down (ueaj/model/mlp.py:90)
    ("bnd,dhik->bnhik", (2, 3, 32), (32, 4, 2, 16)),  # attention q (ueaj/model/soft_attn.py:100)
    ("bnd,dhk->bnhk", (2, 3, 32), (32, 4, 16)),       # attention k / v (ueaj/model/soft_attn.py:83)
    ("bnhiv,hivd->bnd", (2, 3, 4, 2, 16), (4, 2, 16, 32)),  # attention o (ueaj/model/soft_attn.py:117)
])
def test_einsum_oracle_matches_torch_einsum(expr, xs, ws):
    rng = np.random.default_rng(3)
    x = path.bf16_normal(rng, xs)
    w = path.bf16_normal(rng, ws, 0.2)
    y, qx, qw = path.einsum_fp8(expr, x, w)
    ref = torch.einsum(expr, torch.from_numpy(qx.deq()), torch.from_numpy(qw.deq())).numpy()
    ref = fp8.f32_to_bf16_bits(ref.astype(np.float32) * path.alpha_of(qx, qw))
    assert (y == ref).all()
    dy = path.bf16_normal(rng, y.shape, 1e-2)
    dx, dw = path.einsum_fp8_backward(expr, qx, qw, dy)
    xt = torch.from_numpy(qx.deq()).requires_grad_(True)
    wt = torch.from_numpy(qw.deq()).requires_grad_(True)
    qd = path.quant(dy, fp8.E5M2)
    torch.einsum(expr, xt, wt).backward(torch.from_numpy(qd.deq()))
    assert (dx == fp8.f32_to_bf16_bits(xt.grad.numpy().astype(np.float32) * path.alpha_of(qd, qw))).all()
    assert (dw == fp8.f32_to_bf16_bits(wt.grad.numpy().astype(np.float32) * path.alpha_of(qx, qd))).all()


def test_gating_backward_matches_autograd():
    rng = np.random.default_rng(4)
    u = path.bf16_normal(rng, (512,), 2.0)
    g = path.bf16_normal(rng, (512,), 2.0)
    dh = rng.standard_normal(512).astype(np.float32)
    du, dg = path.dswiglu(dh, u, g)
    ut = torch.from_numpy(fp8.bf16_bits_to_f32(u).astype(np.float64)).requires_grad_(True)
    gt = torch.from_numpy(fp8.bf16_bits_to_f32(g).astype(np.float64)).requires_grad_(True)
    (ut * (gt * torch.sigmoid(gt))).backward(torch.from_numpy(fp8.round_bf16(dh).astype(np.float64)))
    rel = lambda a, b: np.abs(a - b).max() / np.abs(b).max()  # noqa: E731
    assert rel(fp8.bf16_bits_to_f32(du), ut.grad.numpy()) < 8e-3
    assert rel(fp8.bf16_bits_to_f32(dg), gt.grad.numpy()) < 8e-3


def test_golden_fixtures_reproduce():
    """The committed vectors equal what the oracle computes now (bit-exact)."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_golden", GOLDEN.parent / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    fresh = mod.build()
    stored = np.load(GOLDEN)
    assert sorted(stored.files) == sorted(fresh)
    for k in stored.files:
        a, b = stored[k], fresh[k]
        if a.dtype == np.float32:
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), k
        else:
            assert np.array_equal(a, b), k


def test_threaded_passes_equal_numpy():
    """The CPU baseline's threaded element-wise passes (fp8.THREADED) give the numpy bits:
    bf16 -> f32 and the RNE f32 -> bf16 rounding on every bf16 pattern and on random f32 values
    (ties included), fp8 -> f32 on all 256 codes of both formats, and a whole oracle GMLP step."""
    allb = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    rng = np.random.default_rng(4)
    f = rng.standard_normal(200_000).astype(np.float32) * np.float32(3e3)
    ties = (fp8.bf16_bits_to_f32(allb[:30000]).view(np.uint32) | np.uint32(0x8000)).view(np.float32)
    f = np.concatenate([f, ties[np.isfinite(ties)], np.array([0.0, -0.0, 3.4e38, -1e-40], np.float32)])
    ref_up = fp8.bf16_bits_to_f32(allb)
    ref_down = fp8.f32_to_bf16_bits(f)
    ref_codes = {fmt: fp8.fp8_to_f64(np.arange(256, dtype=np.uint8), fmt).astype(np.float32) for fmt in (0, 1)}
    x = path.bf16_normal(rng, (64, 48))
    wf = path.bf16_normal(rng, (2, 48, 80), 48 ** -0.5)
    wd = path.bf16_normal(rng, (80, 48), 80 ** -0.5)
    dy = path.bf16_normal(rng, (64, 48), 1e-3)
    y_ref, saved = path.gmlp_forward(x, wf, wd, acc=np.float32)
    g_ref = path.gmlp_backward(dy, saved, acc=np.float32)
    fp8.THREADED = True
    try:
        up = fp8.bf16_bits_to_f32(allb)
        assert np.array_equal(up.view(np.uint32), ref_up.view(np.uint32))
        assert np.array_equal(fp8.f32_to_bf16_bits(f), ref_down)
        for fmt in (0, 1):
            got = fp8.fp8_to_f32_threaded(np.arange(256, dtype=np.uint8), fmt)
            assert np.array_equal(np.isnan(got), np.isnan(ref_codes[fmt]))
            fin = ~np.isnan(got)
            assert np.array_equal(got[fin].view(np.uint32), ref_codes[fmt][fin].view(np.uint32))
        y, saved2 = path.gmlp_forward(x, wf, wd, acc=np.float32)
        g = path.gmlp_backward(dy, saved2, acc=np.float32)
    finally:
        fp8.THREADED = False
    assert np.array_equal(y, y_ref)
    for k in ("dx", "dwf", "dwd"):
        assert np.array_equal(g[k], g_ref[k]), k


def test_norm_oracle_against_float64():
    """The restated RMSNorm (fixed summation order, 1 / sqrt) is within one bf16 rounding of a
    float64 evaluation of the reference formula, for every scale mode."""
    from oracle import norm
    rng = np.random.default_rng(9)
    x = path.bf16_normal(rng, (37, 1000), 3.0)
    xs = fp8.bf16_bits_to_f32(x).astype(np.float64)
    r64 = 1.0 / np.sqrt((xs ** 2).mean(-1, keepdims=True) + 1e-6)
    for scale, centered in ((None, False), (path.bf16_normal(rng, (1000,), 0.5), False),
                            (path.bf16_normal(rng, (1000,), 0.5), True), (path.bf16_normal(rng, (1,)), False),
                            (path.bf16_normal(rng, (1,)), True)):
        y, r = norm.rmsnorm(x, scale, centered, 1e-6)
        w = 1.0 if scale is None else fp8.bf16_bits_to_f32(scale).astype(np.float64)
        w = 1.0 + w if centered else w
        ref = xs * r64 * w
        got = fp8.bf16_bits_to_f32(y).astype(np.float64)
        assert np.allclose(r, r64[:, 0], rtol=1e-6)
        assert np.all(np.abs(got - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-30)


def test_norm_oracle_summation_order():
    """row_sumsq follows the kernel's order exactly: equal to a per-lane loop written out."""
    from oracle import norm
    rng = np.random.default_rng(10)
    x = (rng.standard_normal((3, 300)) * 10).astype(np.float32)
    got = norm.row_sumsq(x)
    for r in range(3):
        lanes = []
        for lane in range(32):
            acc = np.float32(0)
            for c in range(lane, 38, 32):
                for j in range(8):
                    e = 8 * c + j
                    v = x[r, e] if e < 300 else np.float32(0)
                    acc = np.float32(acc + np.float32(v * v))
            lanes.append(acc)
        for o in (16, 8, 4, 2, 1):
            lanes = [np.float32(lanes[i] + lanes[i ^ o]) for i in range(32)]
        assert got[r] == lanes[0]


def test_norm_backward_oracle_matches_autograd():
    """The float64 RMSNorm derivative against torch autograd of the same formula."""
    from oracle import norm
    rng = np.random.default_rng(11)
    x = path.bf16_normal(rng, (5, 64))
    g = path.bf16_normal(rng, (5, 64))
    for scale, centered in ((path.bf16_normal(rng, (64,), 0.5), False), (path.bf16_normal(rng, (64,), 0.5), True),
                            (path.bf16_normal(rng, (1,)), False), (None, False)):
        _, r = norm.rmsnorm(x, scale, centered)
        dx, dw = norm.rmsnorm_backward(x, scale, centered, r, g)
        xt = torch.tensor(fp8.bf16_bits_to_f32(x), dtype=torch.float64, requires_grad=True)
        st = None
        if scale is not None:
            st = torch.tensor(fp8.bf16_bits_to_f32(scale), dtype=torch.float64, requires_grad=True)
        rr = torch.rsqrt((xt ** 2).mean(-1, keepdim=True) + 1e-6)
        w = 1.0 if st is None else (1.0 + st if centered else st)
        (xt * rr * w).backward(torch.tensor(fp8.bf16_bits_to_f32(g), dtype=torch.float64))
        # the oracle takes r from the f32 forward; the bound allows for that rounding
        ref_dx = xt.grad.numpy()
        assert np.allclose(dx, ref_dx, rtol=1e-5, atol=1e-5 * np.abs(ref_dx).max())
        if scale is not None:
            ref_dw = st.grad.numpy().reshape(-1)
            assert np.allclose(dw, ref_dw, rtol=1e-5, atol=1e-5 * np.abs(ref_dw).max())
