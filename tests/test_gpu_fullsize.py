"""The bench workload's own sizes (GMLP C4: 16384 tokens, d_model 4096, hidden 14336), checked
through properties that need no CPU oracle at this size:

* quantize: the bytes equal torch's own RNE cast of f32(x) * s (both follow IEEE RNE; no product
  can overflow because s = FMAX / amax), amax equals torch's max |x|, inv_scale = 1 / s;
* the GEMMs: every output of F1 (with the SwiGLU epilogue), F2, B2 (dSwiGLU) and B4 against an
  fp32 product of the same dequantized fp8 operands (TF32 off), with the bf16 tolerance the
  small-size parity tests use, and the epilogue's max|H| / max|dU, dG| equal to the max of its
  own bf16 outputs, bit for bit.
"""
import pytest

from helpers import COS_TOL, REL_TOL

pytestmark = pytest.mark.gpu

T, D, H = 16384, 4096, 14336


def _close(out, ref, what):
    import torch
    out = out.float().reshape(-1)
    ref = ref.float().reshape(-1)
    assert torch.isfinite(out).all(), f"{what}: non-finite output"
    scale = ref.abs().max()
    max_rel = float((out - ref).abs().max() / scale)
    cos = float(torch.dot(out.double(), ref.double()) / (out.double().norm() * ref.double().norm()))
    assert max_rel <= REL_TOL, f"{what}: max relative error {max_rel:.3e}"
    assert cos >= COS_TOL, f"{what}: cosine {cos:.7f}"


def _deq(q):
    return q.q.float() * q.inv_scale


@pytest.fixture(scope="module")
def tensors(cuda):
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator(device=cuda)
    gen.manual_seed(0)
    x = torch.randn((T, D), generator=gen, device=cuda).to(torch.bfloat16)
    wf = (torch.randn((2, D, H), generator=gen, device=cuda) * D ** -0.5).to(torch.bfloat16)
    wd = (torch.randn((H, D), generator=gen, device=cuda) * H ** -0.5).to(torch.bfloat16)
    dy = (torch.randn((T, D), generator=gen, device=cuda) * 1e-3).to(torch.bfloat16)
    return dict(x=x, qx=ops.quantize(x, C.E4M3), qwf=ops.quantize(wf, C.E4M3), qwd=ops.quantize(wd, C.E4M3),
                qdy=ops.quantize(dy, C.E5M2))


@pytest.mark.parametrize("fmt", [0, 1], ids=["e4m3", "e5m2"])
def test_quantize_full_size_matches_torch_cast(cuda, tensors, fmt):
    import torch
    from macrogpt_jax_b200 import ops
    x = tensors["x"]
    fmax = 448.0 if fmt == 0 else 57344.0
    q = ops.quantize(x, fmt)
    amax = x.float().abs().max()
    assert torch.equal(q.amax.reshape(()), amax)
    s = torch.tensor(fmax, device=cuda) / amax
    ref = (x.float() * s).to(ops.FP8_DTYPE[fmt])
    assert torch.equal(q.q.view(torch.uint8), ref.view(torch.uint8))
    assert torch.equal(q.inv_scale.reshape(()), 1.0 / s)


def test_f1_swiglu_full_size(cuda, tensors):
    import torch
    from macrogpt_jax_b200 import ops
    qx, qwf = tensors["qx"], tensors["qwf"]
    ug, hid, amax_h = ops.gmlp_f1(qx, qwf)
    x32 = _deq(qx)
    for i in range(2):
        _close(ug[i], x32 @ _deq(qwf)[i], f"F1 slice {i}")
    u, g = ug[0].float(), ug[1].float()
    _close(hid, u * (g * torch.sigmoid(g)), "H")
    assert float(amax_h) == float(hid.float().abs().max())


def test_f2_and_b4_full_size(cuda, tensors):
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    import torch
    gen = torch.Generator(device=cuda)
    gen.manual_seed(1)
    qh = ops.quantize(torch.randn((T, H), generator=gen, device=cuda).to(torch.bfloat16), C.E4M3)
    _close(ops.gmlp_f2(qh, tensors["qwd"]), _deq(qh) @ _deq(tensors["qwd"]), "F2")
    del qh
    qdug = ops.quantize((torch.randn((2, T, H), generator=gen, device=cuda) * 1e-3).to(torch.bfloat16), C.E5M2)
    dug32, wf32 = _deq(qdug), _deq(tensors["qwf"])
    ref = dug32[0] @ wf32[0].t()
    ref += dug32[1] @ wf32[1].t()
    _close(ops.gmlp_b4(qdug, tensors["qwf"]), ref, "B4")


def test_b2_dswiglu_full_size(cuda, tensors):
    import torch
    from macrogpt_jax_b200 import ops
    gen = torch.Generator(device=cuda)
    gen.manual_seed(2)
    ug = torch.randn((2, T, H), generator=gen, device=cuda).to(torch.bfloat16)
    dug, amax = ops.gmlp_b2(tensors["qdy"], tensors["qwd"], ug)
    dh = (_deq(tensors["qdy"]) @ _deq(tensors["qwd"]).t()).to(torch.bfloat16).float()
    u, g = ug[0].float(), ug[1].float()
    sg = torch.sigmoid(g)
    _close(dug[0], dh * (g * sg), "dU")
    _close(dug[1], dh * u * (sg * (1 + g * (1 - sg))), "dG")
    assert float(amax) == float(dug.float().abs().max())


def _torch_cast_check(src, q, what):
    """q (an ops.Fp8Tensor of src) against torch's own recipe on the same tensor: amax = max|src|,
    s = FMAX / amax (capped at FLT_MAX), codes = torch's RNE cast of f32(src) * s, inv = 1 / s;
    all bit for bit."""
    import torch
    fmax = 448.0 if q.q.dtype == torch.float8_e4m3fn else 57344.0
    amax = src.float().abs().max()
    assert torch.equal(q.amax.reshape(()), amax), f"{what}: amax"
    # tensor / tensor is an IEEE division (a Python float / tensor is reciprocal-then-multiply)
    s = torch.clamp(torch.tensor(fmax, device=src.device) / amax, max=torch.finfo(torch.float32).max)
    assert torch.equal(q.q.view(torch.uint8), (src.float() * s).to(q.q.dtype).view(torch.uint8)), f"{what}: codes"
    assert torch.equal(q.inv_scale.reshape(()), torch.tensor(1.0, device=src.device) / s), f"{what}: inv_scale"


def test_gmlp_step_full_size_against_torch_chain(cuda):
    """One whole GMLP fwd+bwd step at the bench workload's sizes, checked link by link against
    torch in fp32 (TF32 off) on the step's own intermediates: every quantisation (x, Wf, Wd, H,
    dY, [dU, dG]) bit for bit against torch's cast with torch's amax; every contraction against
    an fp32 product of the same dequantised fp8 operands; H and [dU, dG] against the SwiGLU math
    on the step's own U, G.  The sequence of ops is the one ops.gmlp_forward / gmlp_backward
    run, and their outputs (y, dx, dWf, dWd) are checked bit-identical to it.  (A chain that
    re-quantised its own H would not do: a different max|H| by one bf16 ulp changes the scale,
    and two independent fp8 roundings of H differ by ~5% of y per element.)"""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    torch.backends.cuda.matmul.allow_tf32 = False
    gen = torch.Generator(device=cuda)
    gen.manual_seed(7)
    x = torch.randn((T, D), generator=gen, device=cuda).to(torch.bfloat16)
    wf = (torch.randn((2, D, H), generator=gen, device=cuda) * D ** -0.5).to(torch.bfloat16)
    wd = (torch.randn((H, D), generator=gen, device=cuda) * H ** -0.5).to(torch.bfloat16)
    dy = (torch.randn((T, D), generator=gen, device=cuda) * 1e-3).to(torch.bfloat16)
    # the module-level step
    y_m, saved = ops.gmlp_forward(x, wf, wd)
    dx_m, dwf_m, dwd_m = ops.gmlp_backward(dy, saved)
    del saved
    # the same step, op by op
    qx, qwf, qwd = ops.quantize(x, C.E4M3), ops.quantize(wf, C.E4M3), ops.quantize(wd, C.E4M3)
    _torch_cast_check(x, qx, "x")
    _torch_cast_check(wf, qwf, "Wf")
    _torch_cast_check(wd, qwd, "Wd")
    ug, hid, amax_h = ops.gmlp_f1(qx, qwf)
    x32, wf32, wd32 = _deq(qx), _deq(qwf), _deq(qwd)
    for i in range(2):
        _close(ug[i], x32 @ wf32[i], f"F1 slice {i}")
    u, g = ug[0].float(), ug[1].float()
    sg = torch.sigmoid(g)
    _close(hid, u * (g * sg), "H")
    qh = ops.quantize(hid, C.E4M3, amax_h)
    _torch_cast_check(hid, qh, "H")
    y = ops.gmlp_f2(qh, qwd)
    h32 = _deq(qh)
    _close(y, h32 @ wd32, "y")
    qdy = ops.quantize(dy, C.E5M2)
    _torch_cast_check(dy, qdy, "dY")
    dug, amax_dug = ops.gmlp_b2(qdy, qwd, ug)
    dy32 = _deq(qdy)
    dh = (dy32 @ wd32.t()).to(torch.bfloat16).float()
    _close(dug[0], dh * (g * sg), "dU")
    _close(dug[1], dh * u * (sg * (1 + g * (1 - sg))), "dG")
    del dh, u, g, sg
    dwd = ops.gmlp_b1(qh, qdy)
    _close(dwd, h32.t() @ dy32, "dWd")
    del h32
    qdug = ops.quantize(dug, C.E5M2, amax_dug)
    _torch_cast_check(dug, qdug, "[dU, dG]")
    dx = ops.gmlp_b4(qdug, qwf)
    dwf = ops.gmlp_b3(qx, qdug)
    dug32 = _deq(qdug)
    ref_dx = dug32[0] @ wf32[0].t()
    ref_dx += dug32[1] @ wf32[1].t()
    _close(dx, ref_dx, "dx")
    del ref_dx
    for i in range(2):
        _close(dwf[i], x32.t() @ dug32[i], f"dWf slice {i}")
    for a, b, what in ((y_m, y, "y"), (dx_m, dx, "dx"), (dwf_m, dwf, "dWf"), (dwd_m, dwd, "dWd")):
        assert torch.equal(a, b), f"module step and op sequence differ in {what}"
