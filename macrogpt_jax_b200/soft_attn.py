"""The Q/K/V/O projections of `SoftmaxAttention` (ueaj/model/soft_attn.py:20-124) on the FP8
Einsum.  The attention itself (kvax flash attention in the reference, soft_attn.py:186-196)
is not part of this library: `forward` takes it as a callable.

Kept from the reference: the constructor, the projection expressions and canonical weight
layouts ("bnd,dhk->bnhk" for k and v, "bnd,dhik->bnhik" for q, "bnhiv,hivd->bnd" for o with
zero init), their sharding annotations, and the O-sharding choice (soft_attn.py:108-113).

Added: `fused_qkv=True` builds one Einsum "bnd,fdhk->fbnhk" over a stacked [3, d, h, k]
weight (f indexes q, k, v; requires kv_q_ratio == 1), so the three projections run as one
batched FP8 GEMM with one per-tensor scale — the fused QKV Einsum (d -> 3*h*k) of the
attention-projection workload.
"""
from __future__ import annotations

from typing import Callable, Literal, Optional

import torch

from .configurator import config
from .einsum import Einsum, Rngs, zeros_init


@config
class SoftmaxAttention(torch.nn.Module):
    def __init__(self, model_d: int, kq_d: int = 64, kv_heads: Optional[int] = None, kv_q_ratio: int = 1,
                 rope_theta: Optional[float] = 10000.0, window_size: Optional[int] = None,
                 act_fn: Optional[Callable] = None, k: Callable = Einsum, v: Callable = Einsum,
                 q: Callable = Einsum, o: Callable = Einsum, attn_scale: float | Literal["mup", "sp"] = "sp", *,
                 rngs: Rngs, mesh=None, fused_qkv: bool = False, qkv: Callable = Einsum):
        super().__init__()
        if kv_heads is None:
            kv_heads = model_d // kq_d
        self.model_d, self.kq_d, self.v_head_d = model_d, kq_d, kq_d
        self.kv_heads, self.kv_q_ratio = kv_heads, kv_q_ratio
        self.rope_theta, self.window_size, self.act_fn, self.attn_scale = rope_theta, window_size, act_fn, attn_scale
        size_dict = {"d": model_d, "k": kq_d, "v": kq_d, "h": kv_heads, "i": kv_q_ratio, "f": 2}
        self.fused_qkv = fused_qkv
        if fused_qkv:
            if kv_q_ratio != 1:
                raise ValueError("fused_qkv needs kv_q_ratio == 1 (q, k and v of equal width)")
            self.qkv = qkv("bnd,fdhk->fbnhk", size_dict={**size_dict, "f": 3}, batch_dims="f", rngs=rngs,
                           dtype=torch.bfloat16, mesh=mesh, sharding=(None, None, "tensor", None))
        else:
            self.k = k("bnd,dhk->bnhk", size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16, mesh=mesh,
                       sharding=(None, "tensor", None))
            self.v = v("bnd,dhv->bnhv", size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16, mesh=mesh,
                       sharding=(None, "tensor", None))
            self.q = q("bnd,dhik->bnhik", size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16, mesh=mesh,
                       sharding=(None, "tensor", None, None))
        tensor = getattr(mesh, "shape", {}).get("tensor", 1) if mesh is not None else 1
        if mesh is not None and kv_q_ratio * kq_d * (kv_heads // tensor) > model_d:
            down_shards = ("tensor", None, None, None)  # down-project first, then reduce
        else:
            down_shards = (None, None, None, "tensor")  # attention first, then ring matmul
        self.o = o("bnhiv,hivd->bnd", initializer=zeros_init, size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16,
                   mesh=mesh, sharding=down_shards)

    def project_qkv(self, x: torch.Tensor):
        """q [b, n, h, i, k], k [b, n, h, k], v [b, n, h, v]."""
        if self.fused_qkv:
            qkv = self.qkv(x)  # [3, b, n, h, k]
            b, n = x.shape[:2]
            q = qkv[0].reshape(b, n, self.kv_heads, 1, self.kq_d)
            return q, qkv[1], qkv[2]
        return self.q(x), self.k(x), self.v(x)

    def project_out(self, attn: torch.Tensor) -> torch.Tensor:
        """attn [b, n, h, i, v] -> [b, n, d]."""
        return self.o(attn)

    def forward(self, x: torch.Tensor, attention: Optional[Callable] = None) -> torch.Tensor:
        if attention is None:
            raise NotImplementedError("the attention kernel is not part of this library; pass "
                                      "attention(q, k, v) -> [b, n, h, i, v]")
        q, k, v = self.project_qkv(x)
        return self.project_out(attention(q, k, v))
