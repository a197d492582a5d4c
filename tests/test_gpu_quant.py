"""amax + quantize kernels vs the oracle: bit-exact codes, amax and inverse scale."""
import numpy as np
import pytest

from oracle import fp8 as ofp8
from oracle.path import bf16_normal

from helpers import bits_to_torch_bf16, torch_fp8_to_codes

pytestmark = pytest.mark.gpu


def _run(x_bits, fmt, cuda, offset=0):
    import torch
    from macrogpt_jax_b200 import ops
    n = x_bits.size
    buf = bits_to_torch_bf16(np.concatenate([np.zeros(offset, np.uint16), x_bits.reshape(-1)]), cuda)
    x = buf[offset:]
    # Call through the C ABI with an unaligned view when offset != 0 (scalar kernels).
    from macrogpt_jax_b200 import _capi as C
    q = torch.empty(n + 16, dtype=torch.uint8, device=cuda)[offset:offset + n] if offset else \
        torch.empty(n, dtype=torch.uint8, device=cuda)
    amax = torch.empty(1, dtype=torch.float32, device=cuda)
    inv = torch.empty(1, dtype=torch.float32, device=cuda)
    C.amax_quant(x.data_ptr(), n, fmt, q.data_ptr(), amax.data_ptr(), inv.data_ptr(),
                 torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return q.cpu().numpy(), amax.cpu().numpy().view(np.uint32)[0], inv.cpu().numpy().view(np.uint32)[0]


def _check(x_bits, fmt, cuda, offset=0):
    codes, amax_u, inv_u = _run(x_bits, fmt, cuda, offset)
    rc, ramax, rinv = ofp8.quantize_bits(x_bits.reshape(-1), fmt)
    assert amax_u == np.array([ramax], np.float32).view(np.uint32)[0]
    if np.isnan(rinv):  # NaN amax: any NaN pattern (GPUs produce the canonical 0x7FFFFFFF)
        assert np.isnan(np.array([inv_u], np.uint32).view(np.float32)[0])
    else:
        assert inv_u == np.array([rinv], np.float32).view(np.uint32)[0]
    mism = np.nonzero(codes != rc)[0]
    assert mism.size == 0, f"{mism.size} code mismatches, first at {mism[:5]}: gpu {codes[mism[:5]]} ref {rc[mism[:5]]}"


@pytest.mark.parametrize("fmt", [ofp8.E4M3, ofp8.E5M2])
@pytest.mark.parametrize("n", [0, 1, 7, 15, 16, 17, 1000, 65539, 4_000_037])
def test_quant_random(cuda, fmt, n):
    rng = np.random.default_rng(n)
    _check(bf16_normal(rng, (n,), std=3.0), fmt, cuda)


@pytest.mark.parametrize("fmt", [ofp8.E4M3, ofp8.E5M2])
@pytest.mark.parametrize("offset", [1, 3])
def test_quant_unaligned(cuda, fmt, offset):
    rng = np.random.default_rng(7)
    _check(bf16_normal(rng, (10007,)), fmt, cuda, offset)


@pytest.mark.parametrize("fmt", [ofp8.E4M3, ofp8.E5M2])
def test_quant_all_bf16_patterns(cuda, fmt):
    """Every finite bf16 pattern in one tensor (huge dynamic range: most underflow)."""
    allb = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    finite = (allb & 0x7F80) != 0x7F80
    _check(allb[finite], fmt, cuda)


@pytest.mark.parametrize("fmt", [ofp8.E4M3, ofp8.E5M2])
@pytest.mark.parametrize("case", ["zeros", "tiny", "nan", "inf", "maxbf16", "neg_zero"])
def test_quant_edges(cuda, fmt, case):
    rng = np.random.default_rng(3)
    x = bf16_normal(rng, (4099,))
    if case == "zeros":
        x[:] = 0
    elif case == "tiny":       # denormal amax: FMAX/amax overflows; s is capped at FLT_MAX
        x = (rng.integers(0, 3, 4099).astype(np.uint16)) | (rng.integers(0, 2, 4099).astype(np.uint16) << 15)
    elif case == "nan":
        x[17] = 0x7FC0
    elif case == "inf":
        x[5] = 0xFF80
    elif case == "maxbf16":
        x[9] = 0x7F7F
    elif case == "neg_zero":
        x[:] = 0x8000
    _check(x, fmt, cuda)


def test_quant_ops_wrapper(cuda):
    """ops.quantize on a multi-dimensional tensor and with an externally supplied amax."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(11)
    xb = bf16_normal(rng, (3, 257, 96))
    x = bits_to_torch_bf16(xb, cuda)
    qt = ops.quantize(x, ops.C.E5M2)
    rc, ramax, rinv = ofp8.quantize_bits(xb.reshape(-1), ofp8.E5M2)
    assert qt.q.shape == x.shape and qt.q.dtype == torch.float8_e5m2
    assert (torch_fp8_to_codes(qt.q).reshape(-1) == rc).all()
    half_amax = torch.tensor([float(ramax) / 2], dtype=torch.float32, device=cuda)
    qt2 = ops.quantize(x, ops.C.E4M3, half_amax)
    rc2, _, rinv2 = ofp8.quantize_bits(xb.reshape(-1), ofp8.E4M3, np.float32(float(ramax) / 2))
    assert (torch_fp8_to_codes(qt2.q).reshape(-1) == rc2).all()
    assert qt2.inv_scale.item() == float(rinv2)


@pytest.mark.parametrize("fmt", [ofp8.E4M3, ofp8.E5M2])
@pytest.mark.parametrize("amax", [1e-37, 3e-36, 1e-34])
def test_quant_tiny_amax_stays_finite(cuda, fmt, amax):
    """Normal bf16 tensors whose amax is below FMAX / FLT_MAX: the scale is capped at FLT_MAX,
    so no code is NaN/inf (an uncapped scale would be +inf and turn 0 into NaN), the codes
    match the oracle bit for bit, and code * inv_scale is close to x."""
    rng = np.random.default_rng(5)
    x = bf16_normal(rng, (70001,), std=amax / 4.0)
    x[0] = 0
    _check(x, fmt, cuda)
    codes, _, inv_u = _run(x, fmt, cuda)
    inv = np.array([inv_u], np.uint32).view(np.float32)[0]
    vals = ofp8.fp8_to_f64(codes, fmt)
    assert np.isfinite(vals).all()
    xf = ofp8.bf16_bits_to_f32(x).astype(np.float64)
    deq = vals * np.float64(inv)
    assert np.abs(deq - xf).max() <= 0.13 * np.abs(xf).max()
