"""`SoftmaxAttention` (ueaj/model/soft_attn.py:20-202): the Q/K/V/O projections on the FP8 Einsum,
RoPE on q and k, and the softmax attention of attention.py (the reference calls kvax's flash
attention there, soft_attn.py:186-196).  `forward(x, **kwargs)` follows the reference's __call__:
position_ids (default 0..n-1), query/kv positions and segment ids from kwargs, the 'sp' / 'mup'
or numeric scale; `forward(x, attention)` with a callable attention(q, k, v) -> [b, n, h, i, v]
keeps the projections-only use.

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

import numpy as np
import torch

from .attention import RoPE, softmax_attention
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
        self.rope = RoPE(rope_theta=rope_theta, rope_d=kq_d, value_dtype=torch.bfloat16) if rope_theta else None

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

    def scale(self) -> float:
        if self.attn_scale == "mup":
            return float(np.float32(1.0 / self.kq_d))
        if self.attn_scale == "sp":
            return float(np.float32(1.0 / (self.kq_d ** 0.5)))
        return float(self.attn_scale)

    def forward(self, x: torch.Tensor, attention: Optional[Callable] = None, **kwargs) -> torch.Tensor:
        if attention is not None:
            q, k, v = self.project_qkv(x)
            return self.project_out(attention(q, k, v))
        b, n = x.shape[:2]
        given = kwargs.get("position_ids")
        position_ids = given if given is not None else torch.arange(n, device=x.device)
        q, k, v = self.project_qkv(x)
        if self.rope is not None:
            k = self.rope(k, position_ids=position_ids, rope_freqs=kwargs.get("rope"))
            q = self.rope(q, position_ids=position_ids, rope_freqs=kwargs.get("rope"))
        h, i = q.shape[2], q.shape[3]
        qr = q.reshape(b, n, h * i, self.kq_d)
        # positions 0..n-1 unless given (None lets the kernels use them implicitly)
        qpos = kwargs.get("query_positions", given)
        kpos = kwargs.get("kv_positions", given)
        qseg = kwargs.get("query_segment_ids")
        kseg = kwargs.get("kv_segment_ids", qseg)
        out = softmax_attention(qr, k, v, qpos, qseg, kpos, kseg, kwargs.get("attention_mask"), self.scale())
        out = out.reshape(b, n, h, i, self.kq_d)
        if self.act_fn is not None:
            out = self.act_fn(out)
        return self.project_out(out)
