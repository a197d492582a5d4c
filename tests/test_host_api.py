"""The reference-facing Python API on the CPU: @config / .override() factory injection, Einsum
construction, metadata and GEMM mapping, initializers, and the GMLP fused-path choice."""
import math

import pytest
import torch

from macrogpt_jax_b200.configurator import config, override
from macrogpt_jax_b200.einsum import (Einsum, EinsumMetadata, Rngs, compute_weight_metadata, gemm_plan,
                                      lecun_normal_init, parse_einsum_expr, scaled_normal_init, zeros_init)
from macrogpt_jax_b200.gradutils import LOW_PRECISION, custom_astype, custom_scale, promote_fp8
from macrogpt_jax_b200.mlp import GMLP, MLP, swish

CPU = torch.device("cpu")


# ----------------------------------------------------------------------------- configurator
@config
def _make(a, b=2, *, c=3):
    return (a, b, c)


@config
class _Thing:
    def __init__(self, x, inner=_make, **kw):
        self.x, self.inner, self.kw = x, inner, kw


def test_override_replaces_and_chains():
    f = _make.override(b=5)
    assert f(1) == (1, 5, 3)
    assert f(1, b=9) == (1, 5, 3)  # an override wins over the call-site value
    g = f.override(c=7)
    assert g(0) == (0, 5, 7) and f(0) == (0, 5, 3)


def test_override_validates_keys():
    with pytest.raises(TypeError, match="Invalid override 'zz'"):
        _make.override(zz=1)


class _Plain:
    def __init__(self, x, y=1):
        self.x, self.y = x, y


_Plain = config(_Plain)


def test_class_override_forwards_keywords():
    """Class overrides are constructor keywords (ueaj/utils/configurator.py:152-160)."""
    t = _Thing.override(x=4, extra=1)()
    assert isinstance(t, _Thing) and t.x == 4 and t.kw == {"extra": 1}
    assert _Thing.override(extra=2)(0, extra=3).kw == {"extra": 2}  # the override wins
    with pytest.raises(TypeError):
        _Thing.override(x=4)(0)  # x given twice: positionally and by the override
    t2 = _Thing.override(inner=_make.override(b=11))(1)
    assert t2.inner(0) == (0, 11, 3)
    marker = override(b=11)
    assert _Thing.override(inner=marker)(1).inner == marker  # forwarded as it is
    factory = _Plain.override(zz=1)  # not validated until the constructor runs
    with pytest.raises(TypeError):
        factory(0)
    assert _Plain.override(y=5).override(y=6)(0).y == 6


# ----------------------------------------------------------------------------- Einsum
def test_parse_einsum_expr():
    assert parse_einsum_expr("bnd,idh->ibnh") == ("bnd", "idh", "ibnh")
    with pytest.raises(ValueError):
        parse_einsum_expr("bnd,dh")
    with pytest.raises(ValueError):
        parse_einsum_expr("bnd->bnh")


def test_metadata_of_reference_einsums():
    m = compute_weight_metadata("idh", "ibnh", "i", {"i": 2, "d": 8, "h": 12})
    assert m == EinsumMetadata(canonical_shape=(2, 8, 12), reduced_shape=(2, 8, 12), transpose_axes=[0, 1, 2],
                               batch_ndim=1, reducing_ndim=1, non_reducing_ndim=1, batch_shape=(2,),
                               reducing_shape=(8,), non_reducing_shape=(12,))
    m = compute_weight_metadata("hivd", "bnd", "", {"h": 4, "i": 2, "v": 16, "d": 32})
    assert m.reduced_shape == (128, 32) and m.transpose_axes == [0, 1, 2, 3] and m.reducing_shape == (4, 2, 16)
    m = compute_weight_metadata("dhik", "bnhik", "", {"d": 32, "h": 4, "i": 2, "k": 16})
    assert m.reduced_shape == (32, 128) and m.non_reducing_shape == (4, 2, 16)


@pytest.mark.parametrize("expr,batch,sizes,xshape,want", [
    ("bnd,idh->ibnh", "i", {"i": 2, "d": 8, "h": 12}, (3, 5, 8), (2, (3, 5), 8, 12, (2, 3, 5, 12))),
    ("bnh,hd->bnd", "", {"d": 8, "h": 12}, (3, 5, 12), (1, (3, 5), 12, 8, (3, 5, 8))),
    ("bnhiv,hivd->bnd", "", {"h": 4, "i": 2, "v": 16, "d": 32}, (3, 5, 4, 2, 16), (1, (3, 5), 128, 32, (3, 5, 32))),
    ("bnd,dhik->bnhik", "", {"d": 32, "h": 4, "i": 2, "k": 16}, (3, 5, 32), (1, (3, 5), 32, 128, (3, 5, 4, 2, 16))),
])
def test_gemm_plan(expr, batch, sizes, xshape, want):
    i, w, o = parse_einsum_expr(expr)
    p = gemm_plan(i, w, o, batch, sizes, xshape)
    assert (p.G, p.M_shape, p.K, p.N, p.out_shape) == want


def test_gemm_plan_rejects_non_canonical():
    with pytest.raises(NotImplementedError):
        gemm_plan("bnd", "hd", "bnh", "", {"d": 4, "h": 4}, (1, 1, 4))  # weight not (reducing, non-reducing)


def test_einsum_module_surface():
    e = Einsum("bnd,idh->ibnh", size_dict={"d": 8, "h": 12, "i": 2}, batch_dims="i", rngs=Rngs(0), device=CPU,
               sharding=(None, None, "tensor"))
    assert e.einsum_expr == "bnd,idh->ibnh" and e.w.shape == (2, 8, 12) and e.w.dtype == torch.bfloat16
    assert e.get_einsum_metadata() == {"w": e.metadata}
    e.reshard(mesh="m")
    with pytest.raises(ValueError):
        Einsum("bnd,dh->bnh", size_dict={"d": 4, "h": 4}, rngs=Rngs(0), device=CPU, sharding=("tensor",)).reshard(1)
    with pytest.raises(ValueError, match="CUDA"):  # no CPU path
        e(torch.zeros(1, 3, 8, dtype=torch.bfloat16))


def test_lecun_init_matches_flax_fan_in():
    """variance 1/fan_in with fan_in = shape[-2] * prod(shape[:-2]), truncated at 2 sigma."""
    g = Rngs(1)
    w = lecun_normal_init(64, 96)(g.params(), (2, 256, 512), torch.float32)
    assert abs(w.std().item() - 1 / math.sqrt(512)) / (1 / math.sqrt(512)) < 0.02
    assert w.abs().max().item() <= 2 / math.sqrt(512) / 0.87962566103423978 + 1e-6
    assert (zeros_init(1, 1)(g.params(), (3, 4), torch.bfloat16) == 0).all()
    s = scaled_normal_init(0.5)(1, 1)(g.params(), (200_000,), torch.float32)
    assert abs(s.std().item() - 0.5) < 0.01


def test_rngs_deterministic():
    a = Einsum("bnd,dh->bnh", size_dict={"d": 16, "h": 8}, rngs=Rngs(3), device=CPU)
    b = Einsum("bnd,dh->bnh", size_dict={"d": 16, "h": 8}, rngs=Rngs(3), device=CPU)
    assert torch.equal(a.w, b.w)


# ----------------------------------------------------------------------------- GMLP / MLP
def test_gmlp_fused_detection_and_layout():
    m = GMLP(16, 48, rngs=Rngs(0))
    assert m.fused()
    assert m.fused_proj.w.shape == (2, 16, 48) and m.down_proj.w.shape == (48, 16)
    assert (m.down_proj.w == 0).all()  # zeros_init (ueaj/model/mlp.py:91)
    assert not GMLP(16, 48, activation_fn=torch.nn.functional.gelu, rngs=Rngs(0)).fused()
    m2 = GMLP.override(down_proj=Einsum.override(initializer=scaled_normal_init(0.1)))(16, rngs=Rngs(0))
    assert m2.hidden_d == 64 and m2.fused() and m2.down_proj.w.abs().sum() > 0
    m3 = GMLP.override(fused_proj=Einsum.override(static_scale=2.0))(16, 32, rngs=Rngs(0))
    assert not m3.fused()  # a static scale falls back to the composed path


def test_mlp_builds():
    m = MLP(8, rngs=Rngs(0))
    assert m.up_proj.w.shape == (8, 32) and m.down_proj.w.shape == (32, 8)


def test_attention_projection_layouts():
    from macrogpt_jax_b200.soft_attn import SoftmaxAttention
    a = SoftmaxAttention(64, kq_d=16, kv_heads=4, kv_q_ratio=2, rngs=Rngs(0), k=Einsum.override(device=CPU),
                         v=Einsum.override(device=CPU), q=Einsum.override(device=CPU), o=Einsum.override(device=CPU))
    assert a.k.w.shape == (64, 4, 16) and a.v.w.shape == (64, 4, 16) and a.q.w.shape == (64, 4, 2, 16)
    assert a.o.w.shape == (4, 2, 16, 64) and (a.o.w == 0).all()  # zeros_init (ueaj/model/soft_attn.py:118)
    assert a.q.sharding == (None, "tensor", None, None) and a.o.sharding == (None, None, None, "tensor")
    f = SoftmaxAttention(64, kq_d=16, kv_heads=4, rngs=Rngs(0), fused_qkv=True, qkv=Einsum.override(device=CPU),
                         o=Einsum.override(device=CPU))
    assert f.qkv.w.shape == (3, 64, 4, 16) and f.qkv.einsum_expr == "bnd,fdhk->fbnhk"
    with pytest.raises(ValueError):
        SoftmaxAttention(64, kq_d=16, kv_heads=4, kv_q_ratio=2, rngs=Rngs(0), fused_qkv=True,
                         qkv=Einsum.override(device=CPU), o=Einsum.override(device=CPU))
    with pytest.raises(ValueError, match="CUDA"):  # the attention runs; there is no CPU path
        f(torch.zeros(1, 2, 64))


# ----------------------------------------------------------------------------- gradutils
def test_custom_scale_and_astype_on_cpu():
    x = torch.randn(5, dtype=torch.float32, requires_grad=True)
    y = custom_scale(x, 3.0, scale_forward=True, scale_backward=False)
    y.backward(torch.ones(5))
    assert torch.allclose(y, 3 * x) and torch.allclose(x.grad, torch.ones(5))
    x.grad = None
    y = custom_scale(x, 3.0, scale_forward=False, scale_backward=True)
    y.backward(torch.ones(5))
    assert torch.equal(y, x) and torch.allclose(x.grad, 3 * torch.ones(5))
    x.grad = None
    z = custom_astype(x, torch.bfloat16, cast_forward=True, cast_backward=False)
    assert z.dtype == torch.bfloat16
    with pytest.raises(ValueError, match="GPU"):
        custom_astype(torch.zeros(3, dtype=torch.bfloat16), torch.float8_e4m3fn)


def test_promote_fp8():
    a = torch.zeros(2, dtype=torch.float8_e4m3fn)
    b = torch.zeros(2, dtype=torch.bfloat16)
    c = torch.zeros(2, dtype=torch.float32)
    out = promote_fp8(a, b, c)
    assert out[0].dtype == torch.float32 and out[1].dtype == torch.bfloat16
    assert [t.dtype for t in promote_fp8(a, a)] == [torch.float8_e4m3fn] * 2
    assert torch.float8_e5m2 in LOW_PRECISION
    assert torch.allclose(swish(torch.tensor([0.0, 1.0])), torch.tensor([0.0, 1 / (1 + math.exp(-1))]))


def test_graphed_step_needs_cuda_inputs():
    from macrogpt_jax_b200.graphs import GraphedStep
    with pytest.raises(ValueError, match="CUDA"):
        GraphedStep(lambda t: t, torch.zeros(2))
    with pytest.raises(ValueError, match="CUDA"):
        GraphedStep(lambda: None)
