"""CPU stand-in for the CUDA ops, built on the oracle: lets the tensor-parallel host logic
(sharding, collectives, global scales) run over gloo ranks on a machine without a GPU.
Test infrastructure only."""
from __future__ import annotations

import numpy as np
import torch

from macrogpt_jax_b200.ops import FMT_OF_DTYPE, FP8_DTYPE, Fp8Tensor
from oracle import fp8 as ofp8
from oracle import path as op


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)


def _bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16)


def _q(t: Fp8Tensor) -> op.Q:
    return op.Q(t.q.contiguous().view(torch.uint8).numpy(), FMT_OF_DTYPE[t.q.dtype], np.float32(t.amax.item()),
                np.float32(t.inv_scale.item()))


def _f32(v) -> torch.Tensor:
    return torch.tensor([float(v)], dtype=torch.float32)


class CpuBackend:
    """The backend interface macrogpt_jax_b200.tp.TPContext calls, computed by the oracle."""

    Fp8Tensor = Fp8Tensor

    @staticmethod
    def amax(t: torch.Tensor) -> torch.Tensor:
        return _f32(ofp8.amax_bits(_bits(t)))

    @staticmethod
    def quantize(t: torch.Tensor, fmt: int, amax_t=None) -> Fp8Tensor:
        a = None if amax_t is None else np.float32(amax_t.item())
        r = op.quant(_bits(t), fmt, a)
        q = torch.from_numpy(r.codes.copy()).view(FP8_DTYPE[fmt])
        return Fp8Tensor(q, _f32(r.inv), _f32(r.amax))

    @staticmethod
    def gmlp_f1(qx, qwf):
        a, b = _q(qx), _q(qwf)
        acc = np.einsum("td,idh->ith", a.deq(), b.deq())
        ug = ofp8.f32_to_bf16_bits(acc.astype(np.float32) * op.alpha_of(a, b))
        hid = op.swiglu(ug[0], ug[1])
        return _bf16(ug), _bf16(hid), _f32(ofp8.amax_bits(hid))

    @staticmethod
    def gmlp_f2(qh, qwd):
        return _bf16(op.gemm(_q(qh), _q(qwd), "th", "hd", "td"))

    @staticmethod
    def gmlp_b2(qdy, qwd, ug):
        a, b = _q(qdy), _q(qwd)
        dh = np.einsum("td,hd->th", a.deq(), b.deq()).astype(np.float32) * op.alpha_of(a, b)
        u = _bits(ug)
        du, dg = op.dswiglu(dh, u[0], u[1])
        dug = np.stack([du, dg])
        return _bf16(dug), _f32(ofp8.amax_bits(dug))

    @staticmethod
    def gmlp_b1(qh, qdy):
        return _bf16(op.gemm(_q(qh), _q(qdy), "th", "td", "hd"))

    @staticmethod
    def gmlp_b4(qdug, qwf):
        return _bf16(op.gemm(_q(qdug), _q(qwf), "ith", "idh", "td"))

    @staticmethod
    def gmlp_b3(qx, qdug):
        return _bf16(op.gemm(_q(qx), _q(qdug), "td", "ith", "idh"))
