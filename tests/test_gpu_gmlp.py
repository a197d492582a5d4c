"""FP8 GMLP forward + backward (six contractions, fused gating) vs the oracle."""
import numpy as np
import pytest

from oracle import path as op

from helpers import bf16_bits_to_f64, bits_to_torch_bf16, compare, torch_bf16_to_bits, torch_fp8_to_codes

pytestmark = pytest.mark.gpu


def _inputs(T, d, h, seed=0):
    rng = np.random.default_rng(seed)
    x = op.bf16_normal(rng, (T, d))
    wf = op.bf16_normal(rng, (2, d, h), d ** -0.5)
    wd = op.bf16_normal(rng, (h, d), h ** -0.5)
    dy = op.bf16_normal(rng, (T, d), 1e-3)
    return x, wf, wd, dy


@pytest.mark.parametrize("T,d,h", [(256, 128, 256), (1024, 768, 3072), (384, 256, 640)])
def test_gmlp_fwd_bwd(cuda, T, d, h):
    from macrogpt_jax_b200 import ops
    x, wf, wd, dy = _inputs(T, d, h)
    y, saved = ops.gmlp_forward(bits_to_torch_bf16(x, cuda), bits_to_torch_bf16(wf, cuda),
                                bits_to_torch_bf16(wd, cuda))
    dx, dwf, dwd = ops.gmlp_backward(bits_to_torch_bf16(dy, cuda), saved)
    ry, rs = op.gmlp_forward(x, wf, wd)
    rb = op.gmlp_backward(dy, rs)
    # Operand quantisation of inputs is bit-exact.
    assert (torch_fp8_to_codes(saved[0].q) == rs["qx"].codes).all()
    assert (torch_fp8_to_codes(saved[1].q) == rs["qwf"].codes).all()
    assert (torch_fp8_to_codes(saved[4].q) == rs["qwd"].codes).all()
    compare(bf16_bits_to_f64(torch_bf16_to_bits(saved[2])), bf16_bits_to_f64(rs["ug"]))
    compare(bf16_bits_to_f64(torch_bf16_to_bits(y)), bf16_bits_to_f64(ry))
    compare(bf16_bits_to_f64(torch_bf16_to_bits(dx)), bf16_bits_to_f64(rb["dx"]))
    compare(bf16_bits_to_f64(torch_bf16_to_bits(dwf)), bf16_bits_to_f64(rb["dwf"]))
    compare(bf16_bits_to_f64(torch_bf16_to_bits(dwd)), bf16_bits_to_f64(rb["dwd"]))


def test_gmlp_fwd_bwd_small_workload_full_size(cuda):
    """The small GMLP workload at its own size (8192 tokens, d_model 768, hidden 3072) against
    the oracle; the oracle accumulates in fp32 here (numpy BLAS) to finish in seconds."""
    from macrogpt_jax_b200 import ops
    T, d, h = 8192, 768, 3072
    x, wf, wd, dy = _inputs(T, d, h, seed=3)
    y, saved = ops.gmlp_forward(bits_to_torch_bf16(x, cuda), bits_to_torch_bf16(wf, cuda),
                                bits_to_torch_bf16(wd, cuda))
    dx, dwf, dwd = ops.gmlp_backward(bits_to_torch_bf16(dy, cuda), saved)
    ry, rs = op.gmlp_forward(x, wf, wd, acc=np.float32)
    rb = op.gmlp_backward(dy, rs, acc=np.float32)
    assert (torch_fp8_to_codes(saved[0].q) == rs["qx"].codes).all()
    assert (torch_fp8_to_codes(saved[1].q) == rs["qwf"].codes).all()
    assert (torch_fp8_to_codes(saved[4].q) == rs["qwd"].codes).all()
    for got, ref in ((y, ry), (dx, rb["dx"]), (dwf, rb["dwf"]), (dwd, rb["dwd"])):
        compare(bf16_bits_to_f64(torch_bf16_to_bits(got)), bf16_bits_to_f64(ref))
