"""`TransformerLayer` (ueaj/model/layer.py:11-58) and the fused RMSNorm -> FP8 GMLP block.

The reference layer is  x += attn(attn_norm(x));  x += mlp(mlp_norm(x)).  When the MLP is this
package's fused FP8 GMLP and its norm is this package's RMSNorm, the second half runs as one
autograd node: ufp8_rmsnorm_quant writes the norm's output straight as the e4m3 operand of the
gate/up GEMM (amax and quantisation in the norm's two passes, no bf16 copy of the normalised
activations), and the backward runs the GMLP backward followed by ufp8_rmsnorm_backward.  The
results are the same bits as norm then GMLP, because the GMLP quantises exactly the bf16 tensor
the norm would have returned.

The attention half is SoftmaxAttention: FP8 projections, RoPE and the softmax attention of
attention.py (or a caller's attention callable).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import _capi as C
from . import ops
from .configurator import config
from .einsum import Rngs
from .gradutils import LOW_PRECISION
from .mlp import GMLP
from .rmsnorm import RMSNorm
from .soft_attn import SoftmaxAttention


class _NormGMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, scale, wf, wd, centered, eps):
        qx, rstd = ops.rmsnorm_quant(x2d, scale, centered, eps, C.E4M3)
        y, saved = ops.gmlp_forward_q(qx, wf, wd)
        ctx.saved = saved
        ctx.save_for_backward(x2d, rstd)
        ctx.scale, ctx.centered = scale, centered
        return y

    @staticmethod
    def backward(ctx, dy):
        x2d, rstd = ctx.saved_tensors
        need_dw = ctx.needs_input_grad[2] or ctx.needs_input_grad[3]
        dxn, dwf, dwd = ops.gmlp_backward(dy.to(torch.bfloat16).contiguous(), ctx.saved, True, need_dw)
        ctx.saved = None
        need_ds = ctx.scale is not None and ctx.needs_input_grad[1]
        dx, ds = ops.rmsnorm_backward(x2d, ctx.scale, ctx.centered, rstd, dxn, need_ds)
        dscale = ds.reshape(ctx.scale.shape).to(torch.bfloat16) if need_ds else None
        return dx, dscale, dwf, dwd, None, None


def norm_fusable(norm, mlp) -> bool:
    """True when mlp(norm(x)) can run as the fused RMSNorm -> FP8 GMLP node."""
    return isinstance(norm, RMSNorm) and isinstance(mlp, GMLP) and mlp._tp is None and mlp.fused() and \
        (norm.scale is None or norm.scale.dtype == torch.bfloat16)


def norm_mlp(norm: torch.nn.Module, mlp: torch.nn.Module, x: torch.Tensor) -> torch.Tensor:
    """mlp(norm(x)), fused when norm_fusable(norm, mlp) (same bits either way)."""
    if not norm_fusable(norm, mlp) or x.dtype in LOW_PRECISION:
        return mlp(norm(x))
    lead = x.shape[:-1]
    x2d = x.to(torch.bfloat16).reshape(-1, x.shape[-1]).contiguous()
    wf = mlp.fused_proj.w if mlp.fused_proj.w.dtype == torch.bfloat16 else mlp.fused_proj.w.to(torch.bfloat16)
    wd = mlp.down_proj.w if mlp.down_proj.w.dtype == torch.bfloat16 else mlp.down_proj.w.to(torch.bfloat16)
    y = _NormGMLPFn.apply(x2d, norm.scale, wf, wd, norm.recenter, norm.eps)
    return y.reshape(*lead, mlp.model_d).to(x.dtype)


@config
class TransformerLayer(torch.nn.Module):
    """Transformer layer (ueaj/model/layer.py:11-58): attention and MLP blocks, each behind its
    RMSNorm, with residual connections."""

    def __init__(self, model_d: int, attn: Callable = SoftmaxAttention, mlp: Callable = GMLP,
                 attn_norm: Callable = RMSNorm, mlp_norm: Callable = RMSNorm, *, rngs: Rngs, mesh=None):
        super().__init__()
        self.attn = attn(model_d=model_d, rngs=rngs, mesh=mesh)
        self.mlp = mlp(model_d=model_d, rngs=rngs, mesh=mesh)
        self.attn_norm = attn_norm(model_d=model_d, rngs=rngs, mesh=mesh)
        self.mlp_norm = mlp_norm(model_d=model_d, rngs=rngs, mesh=mesh)
        self.model_d = model_d

    def forward(self, x: torch.Tensor, attention: Optional[Callable] = None, **kwargs) -> torch.Tensor:
        """kwargs as the reference's layer takes them (position_ids, segment ids, rope); `attention`
        replaces the softmax attention with a callable attention(q, k, v) -> [b, n, h, i, v]."""
        x = x + self.attn(self.attn_norm(x), attention, **kwargs)
        return x + norm_mlp(self.mlp_norm, self.mlp, x)
