"""`RMSNorm` (ueaj/model/rmsnorm.py:11-110) on this package's CUDA kernels.

Kept from the reference: the constructor (model_d, scale_mode in 'centered', 'uncentered',
'uncentered_scalar', 'centered_scalar', 'none'; eps; param_dtype; initializer; rngs, mesh,
sharding), the default initialisers (ones for uncentered, zeros for centered), the `scale`
parameter (shape (model_d,) or () for the scalar modes, None for 'none'), the f32 arithmetic
x * rsqrt(mean(x^2) + eps) * scale (or 1 + scale) cast back to the input dtype, and reshard().

The forward runs ufp8_rmsnorm_quant without the fp8 output (bf16 y, per-row rstd kept), the
backward ufp8_rmsnorm_backward.  A layer that feeds the norm's output straight into an FP8
Einsum uses `forward_fp8`, which also quantises y per tensor in the same kernels (layer.py).
"""
from __future__ import annotations

from typing import Callable, Literal, Optional

import torch

from . import ops
from .configurator import config
from .einsum import Rngs

_MODES = {"centered", "uncentered", "centered_scalar", "uncentered_scalar", "none"}


def ones_init(gen, shape, dtype):
    return torch.ones(shape, dtype=dtype)


def zeros_param_init(gen, shape, dtype):
    return torch.zeros(shape, dtype=dtype)


class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, centered, eps):
        lead = x.shape
        x2d = x.to(torch.bfloat16).reshape(-1, lead[-1]).contiguous()
        s = None if scale is None else scale.to(torch.bfloat16)
        y, rstd = ops.rmsnorm(x2d, s, centered, eps)
        ctx.save_for_backward(x2d, rstd)
        ctx.scale, ctx.centered, ctx.lead, ctx.in_dtype = s, centered, lead, x.dtype
        ctx.scale_dtype = None if scale is None else scale.dtype
        return y.reshape(lead).to(x.dtype)

    @staticmethod
    def backward(ctx, dy):
        x2d, rstd = ctx.saved_tensors
        dy2d = dy.to(torch.bfloat16).reshape(x2d.shape).contiguous()
        need_ds = ctx.scale is not None and ctx.needs_input_grad[1]
        dx, ds = ops.rmsnorm_backward(x2d, ctx.scale, ctx.centered, rstd, dy2d, need_ds)
        dscale = None
        if need_ds:
            dscale = ds.reshape(ctx.scale.shape).to(ctx.scale_dtype)
        return dx.reshape(ctx.lead).to(ctx.in_dtype), dscale, None, None


@config
class RMSNorm(torch.nn.Module):
    """Root Mean Square Layer Normalization (ueaj/model/rmsnorm.py:11-84)."""

    def __init__(self, model_d: int,
                 scale_mode: Literal["centered", "uncentered", "uncentered_scalar", "centered_scalar",
                                     "none"] = "uncentered",
                 eps: float = 1e-6, param_dtype: torch.dtype = torch.bfloat16, initializer: Optional[Callable] = None,
                 *, rngs: Rngs, mesh=None, sharding: Optional[str] = "tensor", device=None):
        super().__init__()
        self.eps = eps
        self.recenter = False
        self.sharding = sharding
        self.mesh = mesh
        self.model_d = model_d
        if scale_mode == "none":
            self.scale = None
            return
        if scale_mode not in _MODES:
            raise ValueError(f"Unknown scale_mode: {scale_mode}")
        is_scalar = scale_mode.endswith("_scalar")
        self.recenter = scale_mode.startswith("centered")
        shape = () if is_scalar else (model_d,)
        if initializer is None:
            initializer = zeros_param_init if self.recenter else ones_init
        if device is None:
            device = torch.device("cuda") if torch.cuda.is_available() else torch.device("cpu")
        self.scale = torch.nn.Parameter(initializer(rngs.params(), shape, param_dtype).to(device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return _RMSNormFn.apply(x, self.scale, self.recenter, self.eps)

    def reshard(self, mesh) -> None:
        """Records the mesh (the scale vector is replicated in this package's layouts)."""
        self.mesh = mesh
