"""Precision utilities of the reference, for torch tensors.

  LOW_PRECISION   ueaj/utils/__init__.py:10-16   the fp8 dtype set
  custom_astype   ueaj/utils/gradutils.py:15-54  cast forward values and/or backward grads
  custom_scale    ueaj/utils/gradutils.py:57-93  scale forward values and/or backward grads
  promote_fp8     ueaj/utils/tensorutil.py:127-146

Casts to an fp8 dtype run in this package's quantize kernel with a unit scale (round to
nearest even, ml_dtypes overflow rules); casts between wider dtypes are plain tensor
conversions.
"""
from __future__ import annotations

import torch

from . import _capi as C

LOW_PRECISION = {
    torch.float8_e4m3fn,
    torch.float8_e5m2,
    torch.float8_e4m3fnuz,
    torch.float8_e5m2fnuz,
}

_FP8_FMT = {torch.float8_e4m3fn: C.E4M3, torch.float8_e5m2: C.E5M2}


def cast(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Element-type conversion; bf16 -> fp8 goes through the library's cast kernel."""
    if x.dtype == dtype:
        return x
    if dtype in _FP8_FMT:
        if x.dtype != torch.bfloat16:
            raise TypeError(f"fp8 casts take bfloat16 input, got {x.dtype}")
        if not x.is_cuda:
            raise ValueError("fp8 casts run on the GPU only")
        x = x.contiguous()
        out = torch.empty(x.shape, dtype=dtype, device=x.device)
        C.cast(x.data_ptr(), x.numel(), _FP8_FMT[dtype], out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        return out
    if dtype in LOW_PRECISION:
        raise NotImplementedError(f"casts to {dtype} are not provided")
    return x.to(dtype)


class _CustomAstype(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dtype, cast_forward, cast_backward):
        ctx.dtype, ctx.cast_backward = dtype, cast_backward
        return cast(x, dtype) if cast_forward else x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return (cast(g, ctx.dtype) if ctx.cast_backward else g), None, None, None


def custom_astype(x: torch.Tensor, dtype, cast_forward: bool = True, cast_backward: bool = True) -> torch.Tensor:
    """Casts the forward value and/or the backward gradient to ``dtype``."""
    return _CustomAstype.apply(x, dtype, cast_forward, cast_backward)


class _CustomScale(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, scale_forward, scale_backward):
        ctx.scale, ctx.scale_backward = scale, scale_backward
        return x * scale if scale_forward else x.view_as(x)

    @staticmethod
    def backward(ctx, g):
        return (g * ctx.scale if ctx.scale_backward else g), None, None, None


def custom_scale(x: torch.Tensor, scale: float, scale_forward: bool = True, scale_backward: bool = True):
    """Multiplies the forward value and/or the backward gradient by ``scale``."""
    return _CustomScale.apply(x, scale, scale_forward, scale_backward)


def promote_fp8(*args: torch.Tensor) -> list:
    """Upcasts fp8 arguments to the promoted type of the non-fp8 ones (if any)."""
    common = None
    has_fp8 = False
    for a in args:
        if a.dtype in LOW_PRECISION:
            has_fp8 = True
        elif common is None:
            common = a.dtype
        else:
            common = torch.promote_types(common, a.dtype)
    if not (has_fp8 and common is not None):
        return list(args)
    return [a.to(common) if a.dtype in LOW_PRECISION else a for a in args]
