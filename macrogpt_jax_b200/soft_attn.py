"""`SoftmaxAttention` (ueaj/model/soft_attn.py:20-202): the Q/K/V/O projections on the FP8 Einsum,
RoPE on q and k, and the softmax attention of attention.py (the reference calls kvax's flash
attention there, soft_attn.py:186-196).  `forward(x, **kwargs)` follows the reference's __call__:
position_ids (default 0..n-1), query/kv positions and segment ids from kwargs, the 'sp' / 'mup'
or numeric scale; `forward(x, attention)` with a callable attention(q, k, v) -> [b, n, h, i, v]
keeps the projections-only use.

Kept from the reference: the constructor, the projection expressions and canonical weight
layouts ("bnd,dhk->bnhk" for k and v, "bnd,dhik->bnhik" for q, "bnhiv,hivd->bnd" for o with
zero init), their sharding annotations, and the O-sharding choice (soft_attn.py:108-113).

Tensor parallelism: with a `mesh` whose 'tensor' axis has k > 1 ranks (a DeviceMesh with a
'tensor' dimension, or a ProcessGroup) the block splits over kv heads as the reference's
sharding annotations declare (soft_attn.py:52-75: 'tensor' on h of q/k/v): every rank builds the
full weights, keeps its kv heads of q/k/v and the matching rows of o (the head split of O; the
reference picks O's d axis instead when the attention width per rank is narrower than model_d,
soft_attn.py:108-113, which gives the same sums through a different collective), and forward
takes and returns this rank's token shard [b/k, n, d] (ueaj/model/layer.py:57): x is
all-gathered over tokens, the local heads attend over the full sequences, and the partial
output of o is reduce-scattered back to token shards (copy engines over NVLink, or NCCL).  Every
shard is quantised with the whole logical tensor's scale (Einsum.global_amax), so each rank's
FP8 operands equal the single-GPU ones.  Position and segment ids are taken for the full batch
[b, n] or for the local shard [b/k, n] (then all-gathered).

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
from .gradutils import LOW_PRECISION


def _tensor_size(mesh, group) -> int:
    """Size of the mesh's 'tensor' axis (mesh.shape['tensor'] in the reference's jax Mesh)."""
    if group is not None:
        import torch.distributed as dist
        return dist.get_world_size(group)
    shape = getattr(mesh, "shape", None)
    return shape.get("tensor", 1) if isinstance(shape, dict) else 1


@config
class SoftmaxAttention(torch.nn.Module):
    def __init__(self, model_d: int, kq_d: int = 64, kv_heads: Optional[int] = None, kv_q_ratio: int = 1,
                 rope_theta: Optional[float] = 10000.0, window_size: Optional[int] = None,
                 act_fn: Optional[Callable] = None, k: Callable = Einsum, v: Callable = Einsum,
                 q: Callable = Einsum, o: Callable = Einsum, attn_scale: float | Literal["mup", "sp"] = "sp", *,
                 rngs: Rngs, mesh=None, fused_qkv: bool = False, qkv: Callable = Einsum):
        super().__init__()
        from .tp import TPContext, tensor_group
        group = tensor_group(mesh)
        mk = {"device": torch.device("cpu")} if group is not None else {}
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
                           dtype=torch.bfloat16, mesh=mesh, sharding=(None, None, "tensor", None), **mk)
        else:
            self.k = k("bnd,dhk->bnhk", size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16, mesh=mesh,
                       sharding=(None, "tensor", None), **mk)
            self.v = v("bnd,dhv->bnhv", size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16, mesh=mesh,
                       sharding=(None, "tensor", None), **mk)
            self.q = q("bnd,dhik->bnhik", size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16, mesh=mesh,
                       sharding=(None, "tensor", None, None), **mk)
        tensor = _tensor_size(mesh, group)
        if mesh is not None and kv_q_ratio * kq_d * (kv_heads // tensor) > model_d:
            down_shards = ("tensor", None, None, None)  # down-project first, then reduce
        else:
            down_shards = (None, None, None, "tensor")  # attention first, then ring matmul
        self.o = o("bnhiv,hivd->bnd", initializer=zeros_init, size_dict=size_dict, rngs=rngs, dtype=torch.bfloat16,
                   mesh=mesh, sharding=down_shards, **mk)
        self.rope = RoPE(rope_theta=rope_theta, rope_d=kq_d, value_dtype=torch.bfloat16) if rope_theta else None
        self._tp = None
        if group is not None:
            self._shard(group, TPContext(group))

    def _shard(self, group, tp) -> None:
        """Keeps this rank's kv heads of the projections (see module docstring)."""
        import torch.distributed as dist
        k = dist.get_world_size(group)
        if self.kv_heads % k:
            raise ValueError(f"kv_heads {self.kv_heads} is not divisible by the tensor-parallel size {k}")
        self.o.sharding = ("tensor", None, None, None)  # heads: down-project, then reduce-scatter
        dev = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu")
        for name, operands in (("qkv", ("w", "dout")), ("q", ("w", "dout")), ("k", ("w", "dout")),
                               ("v", ("w", "dout")), ("o", ("x", "w"))):
            e = getattr(self, name, None)
            if e is None:
                continue
            e.reshard(group)
            with torch.no_grad():
                e.w = torch.nn.Parameter(e.w.detach().to(dev))
            e.global_amax = (tp.global_amax, operands)
        self.kv_heads //= k
        self._tp = tp

    def project_qkv(self, x: torch.Tensor):
        """q [b, n, h, i, k], k [b, n, h, k], v [b, n, h, v]."""
        if self.fused_qkv:
            qkv = self.qkv(x)  # [3, b, n, h, k]
            b, n = x.shape[:2]
            q = qkv[0].reshape(b, n, self.kv_heads, 1, self.kq_d)
            return q, qkv[1], qkv[2]
        qx = self._shared_input(x)
        if qx is not None:  # q, k and v read one fp8 copy of x (the same bits each would make)
            return self.q(x, qx), self.k(x, qx), self.v(x, qx)
        return self.q(x), self.k(x), self.v(x)

    def _shared_input(self, x: torch.Tensor):
        """x quantised once for the three projections when they are this package's FP8 Einsums
        with one forward format and x's amax needs no exchange (else None: each quantises)."""
        es = (self.q, self.k, self.v)
        if not all(isinstance(e, Einsum) and type(e).forward is Einsum.forward for e in es) or \
                len({e.fwd_dtype for e in es}) != 1:
            return None
        if any(e.global_amax is not None and "x" in e.global_amax[1] for e in es):
            return None
        if not x.is_cuda or x.numel() == 0 or x.dtype in LOW_PRECISION:
            return None
        from . import ops
        x2 = x.to(torch.bfloat16).reshape(-1, self.model_d).contiguous()
        return ops.quantize(x2, ops.FMT_OF_DTYPE[self.q.fwd_dtype])

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
        if self._tp is None:
            return self._attend(x, attention, **kwargs)
        from .tp import gather_rows, scatter_rows
        tp = self._tp
        bl = x.shape[0]
        ids = {}
        for key in ("position_ids", "query_positions", "kv_positions", "query_segment_ids", "kv_segment_ids"):
            t = kwargs.get(key)
            if isinstance(t, torch.Tensor) and t.dim() == 2 and t.shape[0] == bl and tp.world > 1:
                t = tp.all_gather_rows(t.to(x.device))
            ids[key] = t
        x_full = gather_rows(x.to(torch.bfloat16).contiguous(), tp)
        y_partial = self._attend(x_full, attention, **{**kwargs, **{k: v for k, v in ids.items() if v is not None}})
        return scatter_rows(y_partial.contiguous(), tp)

    def _attend(self, x: torch.Tensor, attention: Optional[Callable] = None, **kwargs) -> torch.Tensor:
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
