"""`GMLP` and `MLP` (ueaj/model/mlp.py:13-115) on top of the FP8 Einsum.

When both GMLP projections are this package's FP8 Einsum and the activation is swish (the
reference default), the whole block runs as gmlp_forward / gmlp_backward: the fused gate/up
contraction writes U, G and H = U * swish(G) from one GEMM epilogue, and the backward fuses
the gating's derivative into the dH epilogue.  Otherwise the block is composed from the
projections exactly as the reference writes it.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch

from . import ops
from .configurator import config
from .einsum import Einsum, Rngs, zeros_init
from .gradutils import LOW_PRECISION


def swish(x: torch.Tensor) -> torch.Tensor:
    """nnx.swish: x * sigmoid(x)."""
    return x * torch.sigmoid(x)


class _GMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x2d, wf, wd):
        y, saved = ops.gmlp_forward(x2d, wf, wd)
        ctx.saved = saved
        return y

    @staticmethod
    def backward(ctx, dy):
        need_dx = ctx.needs_input_grad[0]
        need_dw = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        dx, dwf, dwd = ops.gmlp_backward(dy.to(torch.bfloat16).contiguous(), ctx.saved, need_dx, need_dw)
        ctx.saved = None
        return dx, dwf, dwd


def _is_fp8_einsum(m) -> bool:
    return isinstance(m, Einsum) and m.static_scale is None and m.fwd_dtype == torch.float8_e4m3fn \
        and m.bwd_dtype == torch.float8_e5m2


@config
class MLP(torch.nn.Module):
    """up -> activation -> down (ueaj/model/mlp.py:13-56)."""

    def __init__(self, model_d: int, hidden_d: Optional[int] = None, act_fn: Callable = swish,
                 param_dtype: torch.dtype = torch.bfloat16, up_proj: Callable = Einsum,
                 down_proj: Callable = Einsum, *, rngs: Rngs, mesh=None):
        super().__init__()
        hidden_d = 4 * model_d if hidden_d is None else hidden_d
        size_dict = {"d": model_d, "h": hidden_d}
        self.up_proj = up_proj("bnd,dh->bnh", size_dict=size_dict, rngs=rngs, dtype=param_dtype, mesh=mesh,
                               sharding=(None, "tensor"))
        self.down_proj = down_proj("bnh,hd->bnd", initializer=zeros_init, size_dict=size_dict, rngs=rngs,
                                   dtype=param_dtype, mesh=mesh, sharding=("tensor", None))
        self.activation_fn = act_fn

    def forward(self, x):
        return self.down_proj(self.activation_fn(self.up_proj(x)))


@config
class GMLP(torch.nn.Module):
    """Gated MLP: down(up * act(gate)) with a fused [up, gate] projection
    (ueaj/model/mlp.py:59-115)."""

    def __init__(self, model_d: int, hidden_d: Optional[int] = None, activation_fn: Callable = swish,
                 param_dtype: torch.dtype = torch.bfloat16, fused_proj: Callable = Einsum,
                 down_proj: Callable = Einsum, *, rngs: Rngs, mesh=None, tp_backend=None):
        """With a `mesh` whose 'tensor' axis has k > 1 ranks (a DeviceMesh with a 'tensor'
        dimension, or a ProcessGroup), the block is tensor-parallel exactly as the reference's
        sharding annotations declare it (mlp.py:85,96: gate/up split over hidden, down over its
        input): the projection factories build the full weights, every rank keeps its slice,
        `fused_proj` / `down_proj` are the local shards, and forward takes and returns this
        rank's token shard (ueaj/model/layer.py:57), running tp.TPGMLP's NVLink schedule.
        `tp_backend` replaces the CUDA ops there (tests run the host logic on CPU ranks)."""
        super().__init__()
        hidden_d = 4 * model_d if hidden_d is None else hidden_d
        self.activation_fn = activation_fn
        self.model_d, self.hidden_d = model_d, hidden_d
        self._tp = None
        from .tp import TPGMLP, tensor_group
        group = tensor_group(mesh)
        make_kw = {"device": torch.device("cpu")} if group is not None else {}
        fused = fused_proj("bnd,idh->ibnh", size_dict={"d": model_d, "h": hidden_d, "i": 2},
                           batch_dims="i", rngs=rngs, dtype=param_dtype, mesh=mesh,
                           sharding=(None, None, "tensor"), **make_kw)
        down = down_proj("bnh,hd->bnd", initializer=zeros_init, size_dict={"d": model_d, "h": hidden_d},
                         rngs=rngs, dtype=param_dtype, mesh=mesh, sharding=("tensor", None), **make_kw)
        if group is None:
            self.fused_proj, self.down_proj = fused, down
            return
        if not (_is_fp8_einsum(fused) and _is_fp8_einsum(down)) or activation_fn is not swish:
            raise NotImplementedError("the tensor-parallel GMLP runs the fused FP8 block: FP8 Einsum "
                                      "projections with swish gating")
        self._tp = TPGMLP(model_d, hidden_d, swish, param_dtype, rngs=Rngs(0), group=group, backend=tp_backend,
                          full_weights=(fused.w.detach(), down.w.detach()))
        self.fused_proj, self.down_proj = self._tp.fused_proj, self._tp.down_proj

    def shard_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's token block of a full activation (tensor-parallel blocks only)."""
        if self._tp is None:
            raise ValueError("shard_tokens: this GMLP is not tensor-parallel")
        return self._tp.shard_tokens(x)

    def fused(self) -> bool:
        """True when forward runs as the single fused FP8 GMLP (see module docstring)."""
        return self.activation_fn is swish and _is_fp8_einsum(self.fused_proj) and _is_fp8_einsum(self.down_proj)

    def forward(self, x):
        if self._tp is not None:
            return self._tp(x)
        if self.fused() and x.dtype not in LOW_PRECISION:
            lead = x.shape[:-1]
            wf = self.fused_proj.w
            wd = self.down_proj.w
            wf = wf if wf.dtype == torch.bfloat16 else wf.to(torch.bfloat16)
            wd = wd if wd.dtype == torch.bfloat16 else wd.to(torch.bfloat16)
            x2d = x.to(torch.bfloat16).reshape(-1, self.model_d)
            return _GMLPFn.apply(x2d, wf, wd).reshape(*lead, self.model_d)
        up, gate = self.fused_proj(x)
        gate = self.activation_fn(gate)
        if x.dtype not in LOW_PRECISION:
            h = up * gate
        else:  # ueaj/model/mlp.py:108-111
            s = up.abs().amax(dim=(0, 1), keepdim=True) + 1
            h = ((s * up) * gate) / s
        return self.down_proj(h)
