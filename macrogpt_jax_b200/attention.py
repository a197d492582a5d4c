"""RoPE (ueaj/model/rope.py) and the softmax attention that SoftmaxAttention calls
(ueaj/model/soft_attn.py:186-196, kvax 0.1.2's flash_attention), on this package's kernels
(csrc/attn.cu).

  compute_rope_embedding(pos, rope_theta, rope_d, value_dtype)   rope.py:10-20 (bf16 tables)
  RoPE(rope_theta, rope_d, value_dtype)(x, position_ids, rope_freqs)   rope.py:23-104
  softmax_attention(query, key, value, query_positions, query_segment_ids, kv_positions,
                    kv_segment_ids, mask=None, scale=...)   the flash_attention call's arguments

Attention semantics (kvax's, restated; the wheel is not installable here): query position p sees
key position p' of the same sequence iff p' <= p and both have the same non-negative segment id;
a row that sees nothing outputs 0; query head (h, i) attends with key/value head h.  `mask`
(kvax's precomputed block mask) is accepted and not needed: the kernels derive the mask from the
positions and segment ids.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from . import _capi as C
from . import ops
from .configurator import config


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def rope_inv_freq(rope_d: int, rope_theta: float) -> np.ndarray:
    """1 / theta^(j / half) for j < half, in f32 as the reference's jnp expression computes it."""
    half = rope_d // 2
    e = (np.arange(half, dtype=np.float32) / np.float32(half)).astype(np.float32)
    return (np.float32(1.0) / np.power(np.float32(rope_theta), e).astype(np.float32)).astype(np.float32)


def compute_rope_embedding(pos: torch.Tensor, rope_theta: float, rope_d: int, value_dtype=torch.bfloat16):
    """(sin, cos) [..., rope_d / 2] bf16 for positions `pos` (any shape, on the GPU): the angle
    position * inv_freq in f32, sin / cos in f32, rounded to bf16 (rope.py:10-20 with the
    bf16 value dtype SoftmaxAttention uses)."""
    if not pos.is_cuda:
        raise ValueError("compute_rope_embedding: positions must be a CUDA tensor")
    half = rope_d // 2
    p = pos.to(torch.float32).contiguous()
    inv = torch.from_numpy(rope_inv_freq(rope_d, rope_theta)).to(pos.device)
    sin = torch.empty(tuple(pos.shape) + (half,), dtype=torch.bfloat16, device=pos.device)
    cos = torch.empty_like(sin)
    C.rope_table(p.data_ptr(), p.numel(), half, inv.data_ptr(), sin.data_ptr(), cos.data_ptr(), _stream())
    return sin, cos


class _RopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, sin, cos, period):
        x = x.contiguous()
        tokens = x.shape[0] * x.shape[1]
        d = x.shape[-1]
        heads = x.numel() // (tokens * d) if tokens else 1
        out = torch.empty_like(x)
        C.rope(x.data_ptr(), tokens, heads, d, sin.data_ptr(), cos.data_ptr(), period, False, out.data_ptr(),
               _stream())
        ctx.save_for_backward(sin, cos)
        ctx.geom = (tokens, heads, d, period)
        return out

    @staticmethod
    def backward(ctx, dy):
        sin, cos = ctx.saved_tensors
        tokens, heads, d, period = ctx.geom
        dy = dy.to(torch.bfloat16).contiguous()
        dx = torch.empty_like(dy)
        C.rope(dy.data_ptr(), tokens, heads, d, sin.data_ptr(), cos.data_ptr(), period, True, dx.data_ptr(),
               _stream())
        return dx, None, None, None


@config
class RoPE(torch.nn.Module):
    """Rotary position embedding (rope.py:23-104): x [batch, seq, ..., rope_d], rotating the first
    and second halves of the last axis."""

    def __init__(self, rope_theta: float, rope_d: int, value_dtype=torch.float32):
        super().__init__()
        self.rope_theta, self.rope_d, self.value_dtype = rope_theta, rope_d, value_dtype

    def compute_freqs(self, position_ids: torch.Tensor):
        return compute_rope_embedding(position_ids, self.rope_theta, self.rope_d, self.value_dtype)

    def forward(self, x: torch.Tensor, position_ids: Optional[torch.Tensor] = None, rope_freqs=None) -> torch.Tensor:
        if x.dtype != torch.bfloat16:
            raise TypeError(f"RoPE: the kernel rotates bf16 tensors, got {x.dtype}")
        b, n = x.shape[:2]
        if position_ids is not None:
            sin, cos = self.compute_freqs(position_ids.to(x.device))
        elif rope_freqs is not None:
            sin, cos = (t.to(torch.bfloat16) for t in rope_freqs)
        else:
            sin, cos = self.compute_freqs(torch.arange(n, device=x.device, dtype=torch.float32))
        if sin.dim() == 2:        # (seq, half): one table for every batch element
            if sin.shape[0] < n:
                raise ValueError("RoPE: fewer table rows than sequence positions")
            sin, cos, period = sin[:n].contiguous(), cos[:n].contiguous(), n
        elif sin.dim() == 3:      # (batch, seq, half)
            sin, cos, period = sin.contiguous(), cos.contiguous(), b * n
        else:
            raise ValueError(f"RoPE: unexpected table shape {tuple(sin.shape)}")
        return _RopeFn.apply(x, sin, cos, period)


class _AttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, qseg, kseg, qpos, kpos, scale, group):
        b, n, hi, dh = q.shape
        desc = C.AttnDesc(b, n, hi // group, group, dh,
                          qseg.data_ptr() if qseg is not None else None,
                          kseg.data_ptr() if kseg is not None else None,
                          qpos.data_ptr() if qpos is not None else None,
                          kpos.data_ptr() if kpos is not None else None, float(scale), 0)
        fwd, saved_b, bwd = C.attention_workspace(desc)
        dev = q.device
        ws = torch.empty(max(fwd, 1), dtype=torch.uint8, device=dev)
        saved = torch.empty(max(saved_b, 1), dtype=torch.uint8, device=dev)
        out = torch.empty_like(q)
        fl = 2.0 * 2.0 * b * hi * n * n * dh  # QK^T and PV over the full score matrix
        ops._launch("attention_fwd", fl, lambda: C.attention_forward(
            desc, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), saved.data_ptr(), ws.data_ptr(),
            _stream()))
        ctx.save_for_backward(q, k, v, out, saved, qseg, kseg, qpos, kpos)
        ctx.desc, ctx.bwd = desc, bwd
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, saved, *_ = ctx.saved_tensors
        dout = dout.to(torch.bfloat16).contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        ws = torch.empty(max(ctx.bwd, 1), dtype=torch.uint8, device=q.device)
        b, n, hi, dh = q.shape
        fl = 4.0 * 2.0 * b * hi * n * n * dh  # dP, dQ, dK, dV over the full score matrix
        ops._launch("attention_bwd", fl, lambda: C.attention_backward(
            ctx.desc, q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), dout.data_ptr(), saved.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), _stream()))
        return dq, dk, dv, None, None, None, None, None, None


def _ids(t: Optional[torch.Tensor], b: int, n: int, dev) -> Optional[torch.Tensor]:
    if t is None:
        return None
    t = torch.as_tensor(t, device=dev)
    if t.dim() == 1:
        t = t[None, :].expand(b, n)
    return t.to(torch.int32).contiguous()


def softmax_attention(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                      query_positions: Optional[torch.Tensor] = None, query_segment_ids: Optional[torch.Tensor] = None,
                      kv_positions: Optional[torch.Tensor] = None, kv_segment_ids: Optional[torch.Tensor] = None,
                      mask=None, scale: float = 1.0) -> torch.Tensor:
    """query [b, n, h * i, d], key / value [b, n, h, d] (bf16, CUDA) -> [b, n, h * i, d] bf16."""
    del mask  # derived from positions and segment ids
    b, n, hi, dh = query.shape
    h = key.shape[2]
    if key.shape != (b, n, h, dh) or value.shape != key.shape or hi % h:
        raise ValueError(f"softmax_attention: shapes {tuple(query.shape)}, {tuple(key.shape)}, {tuple(value.shape)}")
    q, k, v = (t.to(torch.bfloat16).contiguous() for t in (query, key, value))
    dev = q.device
    qseg = _ids(query_segment_ids, b, n, dev)
    kseg = _ids(kv_segment_ids, b, n, dev) if kv_segment_ids is not None else qseg
    qpos = _ids(query_positions, b, n, dev)
    kpos = _ids(kv_positions, b, n, dev) if kv_positions is not None else qpos
    return _AttentionFn.apply(q, k, v, qseg, kseg, qpos, kpos, scale, hi // h)
