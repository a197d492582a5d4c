"""The output head of the reference's LlamaModel (ueaj/model/model.py:84-97 and get_logits,
140-165): final RMSNorm, the lm_head Einsum "bnd,dv->bnv" (zeros_init, sharding (None, 'tensor'))
and the optional soft cap 15 * tanh(logits / 15), with the next-token loss fused behind it.

`get_logits` computes what the reference's does (norm -> FP8 lm_head -> cap), bf16 logits out.
`token_loss` is the fused path chunked_softmax_cross_entropy takes for this head: one autograd node
that never hands the logits to the caller:
  forward   ufp8_rmsnorm_quant (norm output written straight as the e4m3 GEMM operand), e4m3
            quantisation of the weight, the lm_head GEMM with the XENT epilogue (bf16 logits, soft
            cap, per-row softmax partials), ufp8_xent_combine (lse, masked loss);
  backward  ufp8_xent_backward (fp8 logit gradient, scale from the per-row results), the two FP8
            GEMMs dX = dL W^T and dW = X^T dL, ufp8_rmsnorm_backward.
The logits are kept from the forward for the backward (2 bytes per logit in HBM) instead of being
recomputed, which the reference's rematerialised chunks do (one GEMM of 2 T d V FLOPs fewer).
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import ops
from .configurator import config
from .einsum import Einsum, Rngs, zeros_init
from .rmsnorm import RMSNorm

HEAD_CAP = 15.0  # the constant of ueaj/model/model.py:163


class _HeadXentFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, scale, w, labels, mask, centered, eps, cap, bwd_fmt):
        loss, saved = ops.head_xent_forward(x2d, scale, centered, eps, w, labels, mask, cap)
        ctx.saved = saved
        ctx.save_for_backward(x2d, labels, mask)
        ctx.scale, ctx.centered, ctx.cap, ctx.bwd_fmt = scale, centered, cap, bwd_fmt
        return loss

    @staticmethod
    def backward(ctx, dloss):
        x2d, labels, mask = ctx.saved_tensors
        rstd = ctx.saved[1]
        need_dw = ctx.needs_input_grad[2]
        dxn, dw = ops.head_xent_backward(dloss.to(torch.float32).contiguous(), ctx.saved, labels, mask, ctx.cap,
                                         need_dw, ctx.bwd_fmt)
        ctx.saved = None
        need_ds = ctx.scale is not None and ctx.needs_input_grad[1]
        dx, ds = ops.rmsnorm_backward(x2d, ctx.scale, ctx.centered, rstd, dxn, need_ds)
        dscale = ds.reshape(ctx.scale.shape).to(torch.bfloat16) if need_ds else None
        return dx, dscale, dw, None, None, None, None, None, None


@config
class OutputHead(torch.nn.Module):
    """Final norm + lm_head + soft cap of LlamaModel (ueaj/model/model.py:84-97, 140-165)."""

    def __init__(self, model_d: int, vocab_size: int, norm: Callable = RMSNorm, lm_head: Callable = Einsum,
                 head_cap: Optional[str] = "tanh", *, rngs: Rngs, mesh=None):
        super().__init__()
        if head_cap not in (None, "tanh"):
            raise ValueError(f"head_cap must be None or 'tanh', got {head_cap!r}")
        self.model_d, self.vocab_size, self.head_cap = model_d, vocab_size, head_cap
        self.norm = norm(model_d=model_d, rngs=rngs, mesh=mesh)
        self.lm_head = lm_head("bnd,dv->bnv", size_dict={"d": model_d, "v": vocab_size}, initializer=zeros_init,
                               rngs=rngs, dtype=torch.bfloat16, mesh=mesh, sharding=(None, "tensor"))

    def get_logits(self, activations: torch.Tensor) -> torch.Tensor:
        """LlamaModel.get_logits: norm -> lm_head -> 15 * tanh(logits / 15) (bf16 arithmetic)."""
        logits = self.lm_head(self.norm(activations))
        if self.head_cap == "tanh":
            logits = HEAD_CAP * torch.tanh(logits / HEAD_CAP)
        return logits

    def forward(self, activations: torch.Tensor) -> torch.Tensor:
        return self.get_logits(activations)

    def fused(self) -> bool:
        """True when token_loss can run the fused norm -> FP8 lm_head -> loss node."""
        lm, nm = self.lm_head, self.norm
        return (isinstance(nm, RMSNorm) and (nm.scale is None or nm.scale.dtype == torch.bfloat16) and
                isinstance(lm, Einsum) and lm.einsum_expr == "bnd,dv->bnv" and lm.static_scale is None and
                lm.fwd_dtype == torch.float8_e4m3fn and getattr(lm, "shard", None) is None)

    def token_loss(self, activations: torch.Tensor, targets: torch.Tensor,
                   mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Per-token loss (f32 [batch, seq]) = softmax_cross_entropy(get_logits(a), targets) * mask,
        through the fused node (fused() must hold)."""
        if not self.fused():
            raise ValueError("token_loss: this head is not the fused RMSNorm + FP8 Einsum combination")
        lead = activations.shape[:-1]
        x2d = activations.to(torch.bfloat16).reshape(-1, self.model_d).contiguous()
        labels = targets.reshape(-1).to(torch.int32).contiguous()
        mk = None if mask is None else mask.reshape(-1).to(torch.uint8).contiguous()
        w = self.lm_head.w if self.lm_head.w.dtype == torch.bfloat16 else self.lm_head.w.to(torch.bfloat16)
        cap = HEAD_CAP if self.head_cap == "tanh" else 0.0
        loss = _HeadXentFn.apply(x2d, self.norm.scale, w, labels, mk, self.norm.recenter, self.norm.eps, cap,
                                 ops.FMT_OF_DTYPE[self.lm_head.bwd_dtype])
        return loss.reshape(lead)
