"""RMSNorm fused with fp8 quantisation (ufp8_rmsnorm_quant / ufp8_rmsnorm_backward) against the
oracle's restatement (oracle/norm.py), the RMSNorm module, and the fused RMSNorm -> FP8 GMLP
node against the unfused modules."""
import numpy as np
import pytest

from oracle import fp8 as ofp8
from oracle import norm as onorm
from oracle import path as op

from helpers import bf16_bits_to_f64, bits_to_torch_bf16, compare, torch_bf16_to_bits, torch_fp8_to_codes

pytestmark = pytest.mark.gpu

MODES = {  # scale_mode: (scale shape builder, centered)
    "uncentered": (lambda d: (d,), False),
    "centered": (lambda d: (d,), True),
    "uncentered_scalar": (lambda d: (1,), False),
    "centered_scalar": (lambda d: (1,), True),
    "none": (None, False),
}


def _case(rng, rows, d, mode):
    x = op.bf16_normal(rng, (rows, d), 2.0)
    shape, centered = MODES[mode]
    scale = None if shape is None else op.bf16_normal(rng, shape(d), 0.5)
    return x, scale, centered


def _f32_bits(t):
    return t.detach().cpu().numpy().view(np.uint32)


@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("rows,d", [(1000, 4096), (7, 100), (33, 4100), (0, 64)])
@pytest.mark.parametrize("fmt", [0, 1])
def test_rmsnorm_quant_bit_exact(cuda, mode, rows, d, fmt):
    import torch
    from macrogpt_jax_b200 import _capi as C
    rng = np.random.default_rng(rows * 7 + d)
    x, scale, centered = _case(rng, rows, d, mode)
    xt = bits_to_torch_bf16(x, cuda)
    st = None if scale is None else bits_to_torch_bf16(scale, cuda)
    q = torch.empty((rows, d), dtype=torch.uint8, device=cuda)
    y = torch.empty((rows, d), dtype=torch.bfloat16, device=cuda)
    amax = torch.empty(1, dtype=torch.float32, device=cuda)
    inv = torch.empty(1, dtype=torch.float32, device=cuda)
    rstd = torch.empty(max(rows, 1), dtype=torch.float32, device=cuda)
    C.rmsnorm_quant(xt.data_ptr(), rows, d, d, st.data_ptr() if st is not None else None,
                    0 if scale is None else scale.size, centered, 1e-6, fmt, q.data_ptr(), amax.data_ptr(),
                    inv.data_ptr(), rstd.data_ptr(), y.data_ptr(), d, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    codes, ramax, rinv, ry, rr = onorm.rmsnorm_quant(x, scale, centered, 1e-6, fmt)
    assert (torch_bf16_to_bits(y) == ry).all()
    assert (_f32_bits(rstd[:rows]) == rr.view(np.uint32)).all()
    assert _f32_bits(amax)[0] == np.array([ramax], np.float32).view(np.uint32)[0]
    assert _f32_bits(inv)[0] == np.array([rinv], np.float32).view(np.uint32)[0]
    assert (torch_fp8_to_codes(q) == codes).all()


@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("rows,d", [(1000, 4096), (7, 100), (33, 4100), (300, 8192)])
def test_rmsnorm_backward(cuda, mode, rows, d):
    """dx (bf16) and dscale (f32) against the float64 derivative at the forward's rstd."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(rows + d)
    x, scale, centered = _case(rng, rows, d, mode)
    g = op.bf16_normal(rng, (rows, d), 1e-2)
    xt = bits_to_torch_bf16(x, cuda)
    st = None if scale is None else bits_to_torch_bf16(scale, cuda)
    _, rstd = ops.rmsnorm(xt, st, centered, 1e-6)
    dx, ds = ops.rmsnorm_backward(xt, st, centered, rstd, bits_to_torch_bf16(g, cuda))
    rdx, rdw = onorm.rmsnorm_backward(x, scale, centered, rstd.cpu().numpy(), g)
    compare(bf16_bits_to_f64(torch_bf16_to_bits(dx)), rdx, rel_tol=1e-2)
    if scale is None:
        assert ds is None
    else:
        got = ds.cpu().numpy().astype(np.float64)
        assert np.abs(got - rdw).max() <= 1e-4 * np.abs(rdw).max()


def test_rmsnorm_deterministic(cuda):
    """Two backward passes give the same bits (fixed-order reductions, no atomics)."""
    import torch
    from macrogpt_jax_b200 import ops
    rng = np.random.default_rng(3)
    x, scale, _ = _case(rng, 4096, 4096, "uncentered")
    xt, st = bits_to_torch_bf16(x, cuda), bits_to_torch_bf16(scale, cuda)
    g = bits_to_torch_bf16(op.bf16_normal(rng, (4096, 4096), 1e-2), cuda)
    _, rstd = ops.rmsnorm(xt, st, False, 1e-6)
    a = ops.rmsnorm_backward(xt, st, False, rstd, g)
    b = ops.rmsnorm_backward(xt, st, False, rstd, g)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("mode", ["uncentered", "centered_scalar", "none"])
def test_rmsnorm_module(cuda, mode):
    """RMSNorm module (reference constructor) forward = oracle bits; backward = the op."""
    import torch
    from macrogpt_jax_b200.einsum import Rngs
    from macrogpt_jax_b200.rmsnorm import RMSNorm
    rng = np.random.default_rng(4)
    m = RMSNorm(256, scale_mode=mode, rngs=Rngs(0), device=cuda)
    if m.scale is not None:
        with torch.no_grad():
            m.scale.copy_(bits_to_torch_bf16(op.bf16_normal(rng, (max(1, m.scale.numel()),), 0.5), cuda).reshape(
                m.scale.shape))
    xb = op.bf16_normal(rng, (2, 50, 256))
    x = bits_to_torch_bf16(xb, cuda).requires_grad_(True)
    y = m(x)
    sb = None if m.scale is None else torch_bf16_to_bits(m.scale).reshape(-1)
    ry, r = onorm.rmsnorm(xb.reshape(100, 256), sb, m.recenter, m.eps)
    assert (torch_bf16_to_bits(y).reshape(100, 256) == ry).all()
    gb = op.bf16_normal(rng, (2, 50, 256), 1e-2)
    y.backward(bits_to_torch_bf16(gb, cuda))
    rdx, rdw = onorm.rmsnorm_backward(xb.reshape(100, 256), sb, m.recenter, r, gb.reshape(100, 256))
    compare(bf16_bits_to_f64(torch_bf16_to_bits(x.grad)).reshape(100, 256), rdx, rel_tol=1e-2)
    if m.scale is not None:
        got = m.scale.grad.float().cpu().numpy().reshape(-1).astype(np.float64)
        assert np.abs(got - rdw).max() <= 1e-2 * np.abs(rdw).max()


@pytest.mark.parametrize("T,d,h", [(512, 256, 640), (16384, 4096, 14336)])
def test_norm_gmlp_fused_equals_unfused(cuda, T, d, h):
    """The fused RMSNorm -> FP8 GMLP node gives the same bits as RMSNorm then GMLP: y, dx,
    dWf, dWd and dscale."""
    import torch
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.layer import norm_fusable, norm_mlp
    from macrogpt_jax_b200.mlp import GMLP
    from macrogpt_jax_b200.rmsnorm import RMSNorm
    mlp = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(d ** -0.5)),
                        down_proj=Einsum.override(initializer=scaled_normal_init(h ** -0.5)))(
        model_d=d, hidden_d=h, rngs=Rngs(1))
    norm = RMSNorm(d, rngs=Rngs(2), device=cuda)
    with torch.no_grad():
        norm.scale.copy_((1 + 0.1 * torch.randn(d, device=cuda)).to(torch.bfloat16))
    assert norm_fusable(norm, mlp)
    gen = torch.Generator(device=cuda)
    gen.manual_seed(5)
    x0 = (torch.randn((T, d), generator=gen, device=cuda) * 3).to(torch.bfloat16)
    dy = (torch.randn((T, d), generator=gen, device=cuda) * 1e-3).to(torch.bfloat16)
    outs = []
    for fused in (True, False):
        x = x0.clone().requires_grad_(True)
        y = norm_mlp(norm, mlp, x) if fused else mlp(norm(x))
        y.backward(dy)
        outs.append([y.detach(), x.grad, mlp.fused_proj.w.grad, mlp.down_proj.w.grad, norm.scale.grad])
        for p in list(mlp.parameters()) + list(norm.parameters()):
            p.grad = None
    for a, b, what in zip(outs[0], outs[1], ("y", "dx", "dWf", "dWd", "dscale")):
        assert torch.equal(a, b), what
