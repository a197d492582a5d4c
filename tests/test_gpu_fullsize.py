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
