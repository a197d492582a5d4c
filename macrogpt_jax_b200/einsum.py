"""FP8 `Einsum` layer: the reference's Einsum module (ueaj/model/einsum.py:150-278) with its
contraction running as per-tensor-scaled FP8 GEMMs in this package's sm_100a kernels.

Kept from the reference, so optimizers, LoRA and weight loaders that read these keep
working: the constructor signature, the canonical weight layout
(...batch_dims, reducing_dims, non_reducing_dims), `w`, `metadata`, `einsum_expr`,
`input_expr` / `weight_expr` / `output_expr`, `batch_dims`, `size_dict`, `sharding`,
`static_scale`, `get_einsum_metadata()` and `reshard()`.

Added keyword-only knobs: `fwd_dtype` (operands of the forward contraction, default
float8_e4m3fn), `bwd_dtype` (incoming gradients, default float8_e5m2) and `device`.
"""
from __future__ import annotations

import math
import operator
from dataclasses import dataclass
from functools import reduce
from typing import Callable, Dict, List, Optional, Tuple

import torch

from . import ops
from .configurator import config

# initializer(in_dims, out_dims) -> init(generator, shape, dtype) -> tensor
InitializerFn = Callable[[int, int], Callable]

_TRUNC_STD = 0.87962566103423978  # std of a standard normal truncated to [-2, 2]


def _fans(shape, in_axis=-2, out_axis=-1):
    """fan_in / fan_out the way JAX's variance_scaling computes them."""
    if len(shape) < 2:
        return (shape[0] if shape else 1), (shape[0] if shape else 1)
    receptive = math.prod(shape) // (shape[in_axis] * shape[out_axis])
    return shape[in_axis] * receptive, shape[out_axis] * receptive


class Rngs:
    """Deterministic source of generators for parameter init (stands in for nnx.Rngs)."""

    def __init__(self, params: int = 0, **_):
        self._seed = int(params)
        self._count = 0

    def params(self) -> torch.Generator:
        g = torch.Generator()
        g.manual_seed(self._seed * 1_000_003 + self._count)
        self._count += 1
        return g


def lecun_normal_init(in_dims: int, out_dims: int):
    """LeCun normal as flax's `nnx.initializers.lecun_normal()` defines it: truncated normal
    ([-2, 2] standard deviations) with variance 1 / fan_in, fan_in taken from the weight
    shape with in_axis=-2, out_axis=-1 (ueaj/model/einsum.py:23-37)."""

    def init(gen: torch.Generator, shape, dtype):
        fan_in, _ = _fans(shape)
        t = torch.empty(shape, dtype=torch.float32)
        torch.nn.init.trunc_normal_(t, 0.0, 1.0, -2.0, 2.0, generator=gen)
        return (t * (math.sqrt(1.0 / fan_in) / _TRUNC_STD)).to(dtype)

    return init


def zeros_init(in_dims: int, out_dims: int):
    def init(gen, shape, dtype):
        return torch.zeros(shape, dtype=dtype)

    return init


def scaled_normal_init(scale: float = 0.75) -> InitializerFn:
    def init_fn(in_dims: int, out_dims: int):
        def init(gen, shape, dtype):
            t = torch.empty(shape, dtype=torch.float32)
            t.normal_(0.0, scale, generator=gen)
            return t.to(dtype)

        return init

    return init_fn


@dataclass
class EinsumMetadata:
    """Canonical/reduced weight shapes for optimizers (ueaj/model/einsum.py:67-78)."""
    canonical_shape: Tuple[int, ...]
    reduced_shape: Tuple[int, ...]
    transpose_axes: List[int]
    batch_ndim: int
    reducing_ndim: int
    non_reducing_ndim: int
    batch_shape: Tuple[int, ...]
    reducing_shape: Tuple[int, ...]
    non_reducing_shape: Tuple[int, ...]


def parse_einsum_expr(expr: str) -> Tuple[str, str, str]:
    """"bnd,dh->bnh" -> ("bnd", "dh", "bnh") (ueaj/model/einsum.py:81-94)."""
    sides = expr.split("->")
    if len(sides) != 2:
        raise ValueError(f"Invalid einsum expression: {expr}")
    operands = sides[0].split(",")
    if len(operands) != 2:
        raise ValueError(f"Expected exactly 2 inputs, got {len(operands)}")
    return operands[0].strip(), operands[1].strip(), sides[1].strip()


def _split_weight_dims(weight_expr: str, output_expr: str, batch_dims: str):
    out = set(output_expr)
    batch = tuple(c for c in weight_expr if c in out and c in batch_dims)
    reducing = tuple(c for c in weight_expr if c not in out)
    non_reducing = tuple(c for c in weight_expr if c in out and c not in batch_dims)
    return batch, reducing, non_reducing


def compute_weight_metadata(weight_expr: str, output_expr: str, batch_dims: str,
                            size_dict: dict) -> EinsumMetadata:
    """Same fields and values as ueaj/model/einsum.py:97-147."""
    b, r, n = _split_weight_dims(weight_expr, output_expr, batch_dims)
    bs = tuple(size_dict[c] for c in b)
    rs = tuple(size_dict[c] for c in r)
    ns = tuple(size_dict[c] for c in n)
    prod = lambda t: reduce(operator.mul, t, 1)  # noqa: E731
    return EinsumMetadata(
        canonical_shape=tuple(size_dict[c] for c in weight_expr),
        reduced_shape=bs + (prod(rs), prod(ns)),
        transpose_axes=[weight_expr.index(c) for c in b + r + n],
        batch_ndim=len(b), reducing_ndim=len(r), non_reducing_ndim=len(n),
        batch_shape=bs, reducing_shape=rs, non_reducing_shape=ns,
    )


def gemm_plan(input_expr: str, weight_expr: str, output_expr: str, batch_dims: str, size_dict: dict,
              x_shape) -> ops.EinsumPlan:
    """Maps a canonical Einsum onto out[g] = X[M, K] @ W[g][K, N].

    Supported (every Einsum the reference builds): weight = batch + reducing + non-reducing
    dims in that order, input = token dims + the reducing dims in weight order, output =
    batch dims + token dims + non-reducing dims.  Anything else raises."""
    b, r, n = _split_weight_dims(weight_expr, output_expr, batch_dims)
    tok = tuple(c for c in input_expr if c not in weight_expr)
    if weight_expr != "".join(b + r + n):
        raise NotImplementedError(f"weight '{weight_expr}' is not in (batch, reducing, non-reducing) order")
    if input_expr != "".join(tok + r):
        raise NotImplementedError(f"input '{input_expr}' is not (token dims + reducing dims '{''.join(r)}')")
    if output_expr != "".join(b + tok + n):
        raise NotImplementedError(f"output '{output_expr}' is not (batch + token + non-reducing dims)")
    if len(x_shape) != len(input_expr):
        raise ValueError(f"input rank {len(x_shape)} does not match '{input_expr}'")
    m_shape = tuple(x_shape[: len(tok)])
    k = math.prod(x_shape[len(tok):])
    if k != math.prod(size_dict[c] for c in r):
        raise ValueError(f"input reducing extent {k} does not match the weight")
    g = math.prod(size_dict[c] for c in b)
    nn = math.prod(size_dict[c] for c in n)
    out_shape = tuple(size_dict[c] for c in b) + m_shape + tuple(size_dict[c] for c in n)
    return ops.EinsumPlan(G=g, M_shape=m_shape, K=k, N=nn, out_shape=out_shape)


class _FP8EinsumFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, plan, fwd_fmt, bwd_fmt, static_scale, global_amax=None, qx=None):
        fn, operands = global_amax if global_amax is not None else (None, ())
        out, saved = ops.einsum_forward(plan, x, w, fwd_fmt, static_scale, fn, operands, qx)
        ctx.plan, ctx.bwd_fmt, ctx.static_scale, ctx.saved = plan, bwd_fmt, static_scale, saved
        ctx.global_amax = (fn, operands)
        ctx.x_shape, ctx.w_shape = x.shape, w.shape
        return out

    @staticmethod
    def backward(ctx, dout):
        need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dx, dw = ops.einsum_backward(ctx.plan, dout.to(torch.bfloat16).contiguous(), ctx.saved, ctx.bwd_fmt,
                                     need_dx, need_dw, ctx.static_scale, *ctx.global_amax)
        ctx.saved = None
        return (dx.reshape(ctx.x_shape) if dx is not None else None,
                dw.reshape(ctx.w_shape) if dw is not None else None, None, None, None, None, None, None)


@config
class Einsum(torch.nn.Module):
    """2-operand einsum layer whose contraction runs in FP8 (see module docstring).

    Weight matrix format: (...batch_dims, reducing_dims, non_reducing_dims)."""

    def __init__(
        self,
        expr: str,
        initializer: InitializerFn = lecun_normal_init,
        size_dict: dict = None,
        batch_dims: str = "",
        dtype: torch.dtype = torch.bfloat16,
        static_scale: Optional[float] = None,
        *,
        rngs: Rngs,
        mesh=None,
        sharding: Optional[tuple] = None,
        fwd_dtype: torch.dtype = torch.float8_e4m3fn,
        bwd_dtype: torch.dtype = torch.float8_e5m2,
        device=None,
    ):
        super().__init__()
        self.input_expr, self.weight_expr, self.output_expr = parse_einsum_expr(expr)
        self.batch_dims = batch_dims
        self.size_dict = size_dict
        self.static_scale = static_scale
        self.sharding = sharding
        self.mesh = mesh
        self.shard = None  # (canonical dim, rank, ranks) once reshard() has sliced the weight
        # (amax_fn, operands): operands ("x", "w", "dout") quantised with amax_fn(t) instead of
        # their local amax; a tensor-parallel block sets it so that shards take the whole
        # logical tensor's scale (a MAX over the group).
        self.global_amax = None
        if fwd_dtype not in ops.FMT_OF_DTYPE or bwd_dtype not in ops.FMT_OF_DTYPE:
            raise ValueError("fwd_dtype / bwd_dtype must be float8_e4m3fn or float8_e5m2")
        self.fwd_dtype, self.bwd_dtype = fwd_dtype, bwd_dtype
        self.metadata = compute_weight_metadata(self.weight_expr, self.output_expr, batch_dims, size_dict)
        b, r, n = _split_weight_dims(self.weight_expr, self.output_expr, batch_dims)
        reducing_size = math.prod(size_dict[c] for c in r)
        non_reducing_size = math.prod(size_dict[c] for c in n)
        init = initializer(reducing_size, non_reducing_size)
        w = init(rngs.params(), self.metadata.canonical_shape, dtype)
        if device is None:
            device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
        self.w = torch.nn.Parameter(w.to(device))
        self.einsum_expr = f"{self.input_expr},{self.weight_expr}->{self.output_expr}"
        # Validates that the expression maps onto the GEMM kernels (raises otherwise).
        token_shape = tuple(1 for c in self.input_expr if c not in self.weight_expr)
        gemm_plan(self.input_expr, self.weight_expr, self.output_expr, batch_dims, size_dict,
                  token_shape + tuple(size_dict[c] for c in r))

    def plan(self, x_shape) -> ops.EinsumPlan:
        return gemm_plan(self.input_expr, self.weight_expr, self.output_expr, self.batch_dims, self.size_dict,
                         tuple(x_shape))

    def forward(self, x: torch.Tensor, qx=None) -> torch.Tensor:
        """`qx`: x already quantised to fwd_dtype as [tokens, reducing] (ops.quantize), shared by
        Einsums that read the same input; gradients still flow to x."""
        w = self.w if self.w.dtype == torch.bfloat16 else self.w.to(torch.bfloat16)
        if x.dtype != torch.bfloat16:
            x = x.to(torch.bfloat16)
        return _FP8EinsumFn.apply(x, w, self.plan(x.shape), ops.FMT_OF_DTYPE[self.fwd_dtype],
                                  ops.FMT_OF_DTYPE[self.bwd_dtype], self.static_scale, self.global_amax, qx)

    def get_einsum_metadata(self) -> Dict[str, EinsumMetadata]:
        return {"w": self.metadata}

    def reshard(self, mesh) -> None:
        """Applies the layer's sharding spec on `mesh` (ueaj/model/einsum.py:257-278).

        The reference places the weight under a NamedSharding; here the weight itself becomes
        this rank's shard: along the canonical dimension the spec marks 'tensor', the rank of
        the mesh's tensor axis keeps its contiguous 1/k slice, and `size_dict` and `metadata`
        describe the local shard.  The layer then computes its local part of the contraction:
        a split output dimension gives this rank's output columns, a split reducing dimension
        a partial sum over this rank's slice of the input (the block that owns the layer
        gathers or reduces, as tp.py does for GMLP).  Without a tensor axis of more than one
        rank, or without 'tensor' in the spec, only the mesh is recorded."""
        from .tp import tensor_group
        import torch.distributed as dist
        sharding = self.sharding if self.sharding is not None else (None,) * len(self.metadata.canonical_shape)
        if len(sharding) != len(self.metadata.canonical_shape):
            raise ValueError(f"Sharding spec length {len(sharding)} doesn't match "
                             f"weight dimensions {len(self.metadata.canonical_shape)}")
        self.mesh = mesh
        group = tensor_group(mesh)
        if group is None or "tensor" not in sharding:
            return
        if getattr(self, "shard", None) is not None:
            raise ValueError("reshard: the weight is already sharded")
        dim = sharding.index("tensor")
        k, r = dist.get_world_size(group), dist.get_rank(group)
        size = self.w.shape[dim]
        if size % k:
            raise ValueError(f"reshard: dimension {dim} of size {size} is not divisible by the tensor axis ({k})")
        local = size // k
        letter = self.weight_expr[dim]  # the weight is stored in weight_expr order
        with torch.no_grad():
            self.w = torch.nn.Parameter(self.w.detach().narrow(dim, r * local, local).contiguous())
        self.size_dict = {**self.size_dict, letter: local}
        self.metadata = compute_weight_metadata(self.weight_expr, self.output_expr, self.batch_dims, self.size_dict)
        self.shard = (dim, r, k)


FP8Einsum = Einsum
