"""Device ops of the FP8 contraction path, each a direct call into libufp8 (include/ufp8.h).

torch is used only for device memory, the current stream and autograd plumbing; every
amax, quantisation and contraction below runs in this package's sm_100a kernels.  There is
no CPU path: inputs must be CUDA tensors and a missing library raises.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _capi as C

FP8_DTYPE = {C.E4M3: torch.float8_e4m3fn, C.E5M2: torch.float8_e5m2}
FMT_OF_DTYPE = {torch.float8_e4m3fn: C.E4M3, torch.float8_e5m2: C.E5M2}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class KernelTimer:
    """Optional per-launch CUDA-event timing of this module's kernels, recorded on the
    stream each kernel is launched on.  Install with set_timer(); read after a sync."""

    def __init__(self):
        self.records = []  # (kind, start_event, end_event, work) ; work = FLOPs or bytes

    def wrap(self, kind: str, work: float, fn):
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        self.records.append((kind, s, e, work))

    def summary(self):
        """{kind: (launches, total_ms, total_work)}"""
        out = {}
        for kind, s, e, work in self.records:
            n, ms, w = out.get(kind, (0, 0.0, 0.0))
            out[kind] = (n + 1, ms + s.elapsed_time(e), w + work)
        return out


_timer: KernelTimer | None = None


def set_timer(t: KernelTimer | None) -> None:
    global _timer
    _timer = t


def get_timer() -> KernelTimer | None:
    return _timer


def _launch(kind: str, work: float, fn) -> None:
    if _timer is None:
        fn()
    else:
        _timer.wrap(kind, work, fn)


def _check_bf16_cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not t.is_cuda:
        raise ValueError(f"{name}: expected a CUDA tensor (this library has no CPU path)")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name}: expected bfloat16, got {t.dtype}")
    return t.contiguous()


@dataclass
class Fp8Tensor:
    """fp8 payload with its per-tensor factors (device f32 scalars)."""
    q: torch.Tensor
    inv_scale: torch.Tensor
    amax: torch.Tensor

    @property
    def fmt(self) -> int:
        return FMT_OF_DTYPE[self.q.dtype]


def amax(x: torch.Tensor) -> torch.Tensor:
    x = _check_bf16_cuda(x, "amax")
    out = torch.empty(1, dtype=torch.float32, device=x.device)
    _launch("amax", 2.0 * x.numel(), lambda: C.amax(x.data_ptr(), x.numel(), out.data_ptr(), _stream()))
    return out


def quantize(x: torch.Tensor, fmt: int, amax_t: torch.Tensor | None = None,
             out: torch.Tensor | None = None) -> Fp8Tensor:
    """Per-tensor current scaling: amax (unless given) -> s = FMAX/amax -> fp8(x*s).
    `out` (optional): a contiguous fp8 tensor of x's element count to write q into."""
    x = _check_bf16_cuda(x, "quantize")
    if out is None:
        q = torch.empty(x.shape, dtype=FP8_DTYPE[fmt], device=x.device)
    else:
        if out.dtype != FP8_DTYPE[fmt] or out.numel() != x.numel() or not out.is_contiguous():
            raise ValueError("quantize: `out` must be a contiguous fp8 tensor of the input's size and format")
        q = out
    inv = torch.empty(1, dtype=torch.float32, device=x.device)
    n = x.numel()
    if amax_t is None:
        amax_t = torch.empty(1, dtype=torch.float32, device=x.device)
        _launch("amax", 2.0 * n, lambda: C.amax(x.data_ptr(), n, amax_t.data_ptr(), _stream()))
    # algorithmic bytes of the quantize pass: 2 B read + 1 B written per element
    _launch("quantize", 3.0 * n,
            lambda: C.quantize(x.data_ptr(), n, fmt, amax_t.data_ptr(), q.data_ptr(), inv.data_ptr(), _stream()))
    return Fp8Tensor(q, inv, amax_t)


def operand(t: Fp8Tensor, major: int, ld: int, batch_stride: int = 0, batch_count: int = 1,
            inv_scale: torch.Tensor | None = None) -> C.Operand:
    inv = t.inv_scale if inv_scale is None else inv_scale
    return C.Operand(t.q.data_ptr(), t.fmt, major, ld, batch_stride, batch_count, 0, inv.data_ptr())


def bf16_operand(t: torch.Tensor, major: int, ld: int, batch_stride: int = 0, batch_count: int = 1,
                 batch_group: int = 0) -> C.Operand:
    """A bf16 GEMM operand (tcgen05 kind::f16), no scale factor; `batch_group` > 1: GEMM batch g
    reads slice g / batch_group."""
    if t.dtype != torch.bfloat16 or not t.is_cuda:
        raise ValueError("bf16_operand: expected a CUDA bfloat16 tensor")
    return C.Operand(t.data_ptr(), C.BF16, major, ld, batch_stride, batch_count, batch_group, None)


def gemm(a: C.Operand, b: C.Operand, M: int, N: int, K: int, d: torch.Tensor, ldd: int,
         d_batch_stride: int = 0, batch: int = 1, k_batches: int = 1, epilogue: int = C.EPI_STORE,
         h: torch.Tensor | None = None, ldh: int = 0, ug: torch.Tensor | None = None, ldug: int = 0,
         ug_batch_stride: int = 0, amax_out: torch.Tensor | None = None, rs_slots: int | None = None,
         rs_rank: int = 0, rs_rows_per_rank: int = 0, ag: tuple | None = None,
         xent: tuple | None = None, axpby: tuple | None = None, tile_mask: int = 0) -> None:
    desc = C.GemmDesc()
    desc.M, desc.N, desc.K = M, N, K
    desc.batch, desc.k_batches = batch, k_batches
    desc.a, desc.b = a, b
    desc.d = d.data_ptr() if d is not None else None
    desc.d_dtype = C.OUT_F32 if (d is not None and d.dtype == torch.float32) else C.OUT_BF16
    desc.epilogue = epilogue
    desc.ldd, desc.d_batch_stride = ldd, d_batch_stride
    desc.h = h.data_ptr() if h is not None else None
    desc.ldh = ldh
    desc.ug = ug.data_ptr() if ug is not None else None
    desc.ldug, desc.ug_batch_stride = ldug, ug_batch_stride
    desc.amax_out = amax_out.data_ptr() if amax_out is not None else None
    if rs_slots is not None:
        desc.rs_slots, desc.rs_rank, desc.rs_rows_per_rank = rs_slots, rs_rank, rs_rows_per_rank
    if ag is not None:  # (flags pointer, epoch, rank, rows per rank): A rows arrive by all-gather
        desc.ag_flags, desc.ag_epoch, desc.ag_rank, desc.ag_rows_per_rank = ag
    if xent is not None:  # (stats tensor, pitch in pairs, soft cap): the XENT epilogue's partials
        desc.xent_stats, desc.xent_ld_stats, desc.xent_cap = xent[0].data_ptr(), xent[1], xent[2]
    desc.tile_mask = tile_mask
    if axpby is not None:  # (C tensor, ldc, c batch stride, alpha, beta): D = alpha acc + beta C
        desc.c, desc.ldc, desc.c_batch_stride = axpby[0].data_ptr(), axpby[1], axpby[2]
        desc.alpha, desc.beta = axpby[3], axpby[4]
    n_eff = 2 * N if epilogue == C.EPI_SWIGLU else N
    flops = 2.0 * M * n_eff * K * batch * k_batches
    _launch("gemm", flops, lambda: C.gemm(desc, _stream()))


# ----------------------------------------------------------------------------- Einsum
@dataclass(frozen=True)
class EinsumPlan:
    """GEMM view of a canonical Einsum: out[g] = X[M,K] @ W[g][K,N]."""
    G: int
    M_shape: tuple
    K: int
    N: int
    out_shape: tuple


def einsum_forward(plan: EinsumPlan, x: torch.Tensor, w: torch.Tensor, fwd_fmt: int,
                   alpha: float | None = None, amax_fn=None, amax_operands=(), qx: Fp8Tensor | None = None):
    """Forward of ueaj.model.Einsum (ueaj/model/einsum.py:233-251) in FP8.  `amax_fn(t)` gives
    the amax of the operands named in `amax_operands` ("x", "w"): under tensor parallelism the
    MAX over the group, so that a shard is quantised with the whole logical tensor's scale.
    `qx`: x already quantised ([M, K], fwd_fmt) by the caller, e.g. once for several Einsums that
    share the input."""
    G, K, N = plan.G, plan.K, plan.N
    M = 1
    for s in plan.M_shape:
        M *= s
    x2 = x.reshape(M, K)
    w3 = w.reshape(G, K, N)
    if qx is None:
        qx = quantize(x2, fwd_fmt, amax_fn(x2) if "x" in amax_operands else None)
    elif qx.fmt != fwd_fmt or tuple(qx.q.shape) != (M, K):
        raise ValueError("einsum_forward: the pre-quantised input does not match the expression")
    qw = quantize(w3, fwd_fmt, amax_fn(w3) if "w" in amax_operands else None)
    out = torch.empty((G, M, N), dtype=torch.bfloat16, device=x.device)
    inv_b = qw.inv_scale if alpha is None else qw.inv_scale * alpha
    gemm(operand(qx, C.K_MAJOR, K), operand(qw, C.MN_MAJOR, N, K * N, G, inv_scale=inv_b),
         M, N, K, out, N, M * N, batch=G)
    return out.reshape(plan.out_shape), (qx, qw)


def einsum_backward(plan: EinsumPlan, dout: torch.Tensor, saved, bwd_fmt: int, need_dx: bool, need_dw: bool,
                    alpha: float | None = None, amax_fn=None, amax_operands=()):
    """dX = dOut W^T (summed over weight batch slices) and dW = X^T dOut; `amax_fn` as in
    einsum_forward, for "dout"."""
    qx, qw = saved
    G, K, N = plan.G, plan.K, plan.N
    M = qx.q.shape[0]
    d2 = dout.reshape(G * M, N)
    qd = quantize(d2, bwd_fmt, amax_fn(d2) if "dout" in amax_operands else None)
    dx = dw = None
    if need_dx:
        dx = torch.empty((M, K), dtype=torch.bfloat16, device=dout.device)
        inv_b = qw.inv_scale if alpha is None else qw.inv_scale * alpha
        gemm(operand(qd, C.K_MAJOR, N, M * N, G), operand(qw, C.K_MAJOR, N, K * N, G, inv_scale=inv_b),
             M, K, N, dx, K, k_batches=G)
    if need_dw:
        dw = torch.empty((G, K, N), dtype=torch.bfloat16, device=dout.device)
        gemm(operand(qx, C.MN_MAJOR, K), operand(qd, C.MN_MAJOR, N, M * N, G),
             K, N, M, dw, N, K * N, batch=G)
    return dx, dw


# ----------------------------------------------------------------------------- GMLP
# The six contractions of one GMLP step (ueaj/model/mlp.py:100-115 and the backward JAX
# derives for it).  Shapes: x [T, d], Wf [2, d, h] (index 0 = up, 1 = gate), Wd [h, d].
def gmlp_f1(qx: Fp8Tensor, qwf: Fp8Tensor, ag: tuple | None = None):
    """[U, G] = x Wf with H = U * swish(G) and max|H| from the epilogue.  `ag`: x's row
    blocks arrive by ufp8_tp_ag_push (flags, epoch, rank, rows per rank)."""
    T, d = qx.q.shape
    h = qwf.q.shape[2]
    dev = qx.q.device
    ug = torch.empty((2, T, h), dtype=torch.bfloat16, device=dev)
    hid = torch.empty((T, h), dtype=torch.bfloat16, device=dev)
    amax_h = torch.empty(1, dtype=torch.float32, device=dev)
    gemm(operand(qx, C.K_MAJOR, d), operand(qwf, C.MN_MAJOR, h, d * h, 2), T, h, d, ug, h, T * h,
         epilogue=C.EPI_SWIGLU, h=hid, ldh=h, amax_out=amax_h, ag=ag)
    return ug, hid, amax_h


def gmlp_f2(qh: Fp8Tensor, qwd: Fp8Tensor) -> torch.Tensor:
    """y = H Wd."""
    T, h = qh.q.shape
    d = qwd.q.shape[1]
    y = torch.empty((T, d), dtype=torch.bfloat16, device=qh.q.device)
    gemm(operand(qh, C.K_MAJOR, h), operand(qwd, C.MN_MAJOR, d), T, d, h, y, d)
    return y


def gmlp_b2(qdy: Fp8Tensor, qwd: Fp8Tensor, ug: torch.Tensor, ag: tuple | None = None):
    """dH = dY Wd^T fused with the gating backward -> [dU, dG] and max|dU, dG|.  `ag`: dY's
    row blocks arrive by ufp8_tp_ag_push."""
    T, d = qdy.q.shape
    h = qwd.q.shape[0]
    dev = qdy.q.device
    dug = torch.empty((2, T, h), dtype=torch.bfloat16, device=dev)
    amax_dug = torch.empty(1, dtype=torch.float32, device=dev)
    gemm(operand(qdy, C.K_MAJOR, d), operand(qwd, C.K_MAJOR, d), T, h, d, dug, h, T * h,
         epilogue=C.EPI_DSWIGLU, ug=ug, ldug=h, ug_batch_stride=T * h, amax_out=amax_dug, ag=ag)
    return dug, amax_dug


def gmlp_f2_push(qh: Fp8Tensor, qwd: Fp8Tensor, rs_slots: int, rank: int, rows_per_rank: int) -> None:
    """y partial = H Wd with every row stored into its owner rank's staging slot (RS_PUSH)."""
    T, h = qh.q.shape
    d = qwd.q.shape[1]
    gemm(operand(qh, C.K_MAJOR, h), operand(qwd, C.MN_MAJOR, d), T, d, h, None, d, epilogue=C.EPI_RS_PUSH,
         rs_slots=rs_slots, rs_rank=rank, rs_rows_per_rank=rows_per_rank)


def gmlp_b4_push(qdug: Fp8Tensor, qwf: Fp8Tensor, rs_slots: int, rank: int, rows_per_rank: int) -> None:
    """dx partial = sum_i dUG[i] Wf[i]^T stored into the owners' staging slots (RS_PUSH)."""
    _, T, h = qdug.q.shape
    d = qwf.q.shape[1]
    gemm(operand(qdug, C.K_MAJOR, h, T * h, 2), operand(qwf, C.K_MAJOR, h, d * h, 2), T, d, h, None, d,
         k_batches=2, epilogue=C.EPI_RS_PUSH, rs_slots=rs_slots, rs_rank=rank, rs_rows_per_rank=rows_per_rank)


def gmlp_b1(qh: Fp8Tensor, qdy: Fp8Tensor) -> torch.Tensor:
    """dWd = H^T dY (contraction over tokens; MN-major operands, no transposed copies)."""
    T, h = qh.q.shape
    d = qdy.q.shape[1]
    dwd = torch.empty((h, d), dtype=torch.bfloat16, device=qh.q.device)
    gemm(operand(qh, C.MN_MAJOR, h), operand(qdy, C.MN_MAJOR, d), h, d, T, dwd, d)
    return dwd


def gmlp_b4(qdug: Fp8Tensor, qwf: Fp8Tensor) -> torch.Tensor:
    """dx = sum_i dUG[i] Wf[i]^T (K concatenated over [up, gate])."""
    _, T, h = qdug.q.shape
    d = qwf.q.shape[1]
    dx = torch.empty((T, d), dtype=torch.bfloat16, device=qdug.q.device)
    gemm(operand(qdug, C.K_MAJOR, h, T * h, 2), operand(qwf, C.K_MAJOR, h, d * h, 2), T, d, h, dx, d, k_batches=2)
    return dx


def gmlp_b3(qx: Fp8Tensor, qdug: Fp8Tensor) -> torch.Tensor:
    """dWf[i] = x^T dUG[i]."""
    T, d = qx.q.shape
    h = qdug.q.shape[2]
    dwf = torch.empty((2, d, h), dtype=torch.bfloat16, device=qx.q.device)
    gemm(operand(qx, C.MN_MAJOR, d), operand(qdug, C.MN_MAJOR, h, T * h, 2), d, h, T, dwf, h, d * h, batch=2)
    return dwf


def gmlp_forward(x: torch.Tensor, wf: torch.Tensor, wd: torch.Tensor):
    """FP8 GMLP forward, GMLP.__call__ (ueaj/model/mlp.py:100-115) with the fused gate/up
    Einsum "bnd,idh->ibnh" and its gating fused into one GEMM epilogue.

    x [T, d] bf16, wf [2, d, h] bf16 (index 0 = up, 1 = gate), wd [h, d] bf16.
    Returns y [T, d] bf16 and the tensors the backward needs.
    """
    x = _check_bf16_cuda(x, "x")
    return gmlp_forward_q(quantize(x, C.E4M3), wf, wd)


def gmlp_forward_q(qx: Fp8Tensor, wf: torch.Tensor, wd: torch.Tensor):
    """gmlp_forward from an already quantised input (e4m3 [T, d]), e.g. the fp8 output of
    rmsnorm_quant."""
    if qx.fmt != C.E4M3:
        raise ValueError("gmlp_forward_q: the input must be float8_e4m3fn")
    wf = _check_bf16_cuda(wf, "wf")
    wd = _check_bf16_cuda(wd, "wd")
    qwf = quantize(wf, C.E4M3)
    ug, hid, amax_h = gmlp_f1(qx, qwf)
    qh = quantize(hid, C.E4M3, amax_h)
    qwd = quantize(wd, C.E4M3)
    y = gmlp_f2(qh, qwd)
    return y, (qx, qwf, ug, qh, qwd)


def gmlp_backward(dy: torch.Tensor, saved, need_dx: bool = True, need_dw: bool = True):
    """Backward of gmlp_forward: the four contractions JAX derives for the two Einsums plus
    the gating backward, with e5m2 gradients and e4m3 saved operands."""
    qx, qwf, ug, qh, qwd = saved
    dy = _check_bf16_cuda(dy, "dy")
    qdy = quantize(dy, C.E5M2)
    dug, amax_dug = gmlp_b2(qdy, qwd, ug)
    dwd = gmlp_b1(qh, qdy) if need_dw else None
    qdug = quantize(dug, C.E5M2, amax_dug)
    dx = gmlp_b4(qdug, qwf) if need_dx else None
    dwf = gmlp_b3(qx, qdug) if need_dw else None
    return dx, dwf, dwd


def device_status(clear: bool = True) -> int:
    return C.device_status(clear)


# ----------------------------------------------------------------------------- RMSNorm
# RMSNorm (ueaj/model/rmsnorm.py:68-84) on [rows, d] bf16 activations, alone (bf16 out) or fused
# with the per-tensor fp8 quantisation of its output for the FP8 Einsum that consumes it.
def _norm_scale(scale: torch.Tensor | None):
    if scale is None:
        return None, 0
    s = _check_bf16_cuda(scale.reshape(-1), "rmsnorm scale")
    return s, s.numel()


def rmsnorm(x2d: torch.Tensor, scale: torch.Tensor | None, centered: bool, eps: float):
    """(y bf16 [rows, d], rstd f32 [rows])."""
    x2d = _check_bf16_cuda(x2d, "rmsnorm x")
    rows, d = x2d.shape
    s, slen = _norm_scale(scale)
    y = torch.empty_like(x2d)
    rstd = torch.empty(rows, dtype=torch.float32, device=x2d.device)
    _launch("norm", 4.0 * rows * d, lambda: C.rmsnorm_quant(
        x2d.data_ptr(), rows, d, d, s.data_ptr() if s is not None else None, slen, centered, eps, 0, None, None,
        None, rstd.data_ptr(), y.data_ptr(), d, _stream()))
    return y, rstd


def rmsnorm_quant(x2d: torch.Tensor, scale: torch.Tensor | None, centered: bool, eps: float, fmt: int):
    """RMSNorm fused with the fp8 quantisation of its output: (Fp8Tensor of y, rstd).  The
    algorithmic traffic is 5 B per element (x read twice, fp8 written)."""
    x2d = _check_bf16_cuda(x2d, "rmsnorm x")
    rows, d = x2d.shape
    s, slen = _norm_scale(scale)
    q = torch.empty((rows, d), dtype=FP8_DTYPE[fmt], device=x2d.device)
    amax_t = torch.empty(1, dtype=torch.float32, device=x2d.device)
    inv = torch.empty(1, dtype=torch.float32, device=x2d.device)
    rstd = torch.empty(rows, dtype=torch.float32, device=x2d.device)
    _launch("norm_quant", 5.0 * rows * d, lambda: C.rmsnorm_quant(
        x2d.data_ptr(), rows, d, d, s.data_ptr() if s is not None else None, slen, centered, eps, fmt,
        q.data_ptr(), amax_t.data_ptr(), inv.data_ptr(), rstd.data_ptr(), None, 0, _stream()))
    return Fp8Tensor(q, inv, amax_t), rstd


def rmsnorm_backward(x2d: torch.Tensor, scale: torch.Tensor | None, centered: bool, rstd: torch.Tensor,
                     dy2d: torch.Tensor, need_dscale: bool = True):
    """(dx bf16 [rows, d], dscale f32 [scale elements] or None)."""
    x2d = _check_bf16_cuda(x2d, "rmsnorm x")
    dy2d = _check_bf16_cuda(dy2d, "rmsnorm dy")
    rows, d = x2d.shape
    s, slen = _norm_scale(scale)
    dx = torch.empty_like(x2d)
    dscale = ws = None
    nbytes = 0
    if s is not None and need_dscale:
        dscale = torch.empty(slen, dtype=torch.float32, device=x2d.device)
        nbytes = C.rmsnorm_backward_workspace(rows, d)
        ws = torch.empty(nbytes // 4, dtype=torch.float32, device=x2d.device)
    _launch("norm_bwd", 6.0 * rows * d, lambda: C.rmsnorm_backward(
        x2d.data_ptr(), rows, d, d, s.data_ptr() if s is not None else None, slen, centered, rstd.data_ptr(),
        dy2d.data_ptr(), d, dx.data_ptr(), d, dscale.data_ptr() if dscale is not None else None,
        ws.data_ptr() if ws is not None else None, nbytes, _stream()))
    return dx, dscale


# ----------------------------------------------------------------------------- lm_head + loss
# The output head of LlamaModel.get_logits (ueaj/model/model.py:140-165: final RMSNorm, lm_head
# Einsum "bnd,dv->bnv", optional 15 * tanh(l / 15)) followed by the per-token next-token loss of
# chunked_softmax_cross_entropy (ueaj/opt/next_token_loss.py:99-174).  x [T, d] bf16, w [d, V]
# bf16, labels int32 [T], mask uint8 [T] or None.  The lm_head weight is quantised into a
# [d, Vp] buffer, Vp = V rounded up to 16 (the MN-major operand's 16-byte pitch rule); the
# logits and the fp8 logit gradient use the same pitch.
def _pad16(n: int) -> int:
    return (n + 15) // 16 * 16


def xent_rows(logits: torch.Tensor, labels: torch.Tensor, mask: torch.Tensor | None, V: int | None = None):
    """(lse, loss, qrow) f32 [rows] from bf16 logits [rows, >= V] (ufp8_xent_forward)."""
    if not logits.is_cuda or logits.dtype != torch.bfloat16 or (logits.numel() and logits.stride(1) != 1):
        raise ValueError("xent_rows: logits must be a CUDA bf16 tensor with unit column stride")
    rows = logits.shape[0]
    V = logits.shape[1] if V is None else V
    lse, loss, qrow = (torch.empty(rows, dtype=torch.float32, device=logits.device) for _ in range(3))
    ldl = logits.stride(0) if rows else V  # an empty tensor's strides carry no pitch
    _launch("xent_rows", 2.0 * rows * V, lambda: C.xent_forward(
        logits.data_ptr(), rows, V, ldl, labels.data_ptr(),
        mask.data_ptr() if mask is not None else None, lse.data_ptr(), loss.data_ptr(), qrow.data_ptr(), _stream()))
    return lse, loss, qrow


def xent_grad(logits: torch.Tensor, labels: torch.Tensor, mask: torch.Tensor | None, lse: torch.Tensor,
              qrow: torch.Tensor | None, dloss: torch.Tensor | None, cap: float, fmt: int, V: int | None = None):
    """dlogits from bf16 logits (ufp8_xent_backward): a bf16 [rows, V] tensor for fmt BF16, else an
    Fp8Tensor [rows, Vp] (pitch Vp) with its per-tensor factors."""
    rows = logits.shape[0]
    V = logits.shape[1] if V is None else V
    dev = logits.device
    if fmt == C.BF16:
        out = torch.empty((rows, V), dtype=torch.bfloat16, device=dev)
        ldo, amax_t, inv = V, None, None
    else:
        ldo = _pad16(V)
        out = torch.empty((rows, ldo), dtype=FP8_DTYPE[fmt], device=dev)
        amax_t = torch.empty(1, dtype=torch.float32, device=dev)
        inv = torch.empty(1, dtype=torch.float32, device=dev)
    nbytes = (2.0 + (2.0 if fmt == C.BF16 else 1.0)) * rows * V
    ldl = logits.stride(0) if rows else V
    _launch("xent_grad", nbytes, lambda: C.xent_backward(
        logits.data_ptr(), rows, V, ldl, labels.data_ptr(),
        mask.data_ptr() if mask is not None else None, lse.data_ptr(),
        qrow.data_ptr() if qrow is not None else None, dloss.data_ptr() if dloss is not None else None,
        float(cap), fmt, out.data_ptr(), ldo, amax_t.data_ptr() if amax_t is not None else None,
        inv.data_ptr() if inv is not None else None, _stream()))
    return out if fmt == C.BF16 else Fp8Tensor(out, inv, amax_t)


def quantize_head_weight(w: torch.Tensor) -> Fp8Tensor:
    """e4m3 per-tensor quantisation of the lm_head weight [d, V] into a [d, Vp] buffer."""
    w = _check_bf16_cuda(w, "lm_head w")
    d, V = w.shape
    Vp = _pad16(V)
    if Vp != V:
        w = torch.nn.functional.pad(w, (0, Vp - V))  # zero columns leave amax unchanged
    return quantize(w, C.E4M3)


def head_logits(qx: Fp8Tensor, qw: Fp8Tensor, V: int, cap: float):
    """logits = x W with the XENT epilogue: (logits bf16 [T, Vp] (columns < V valid), stats)."""
    T, d = qx.q.shape
    Vp = qw.q.shape[1]
    groups = (V + 127) // 128
    logits = torch.empty((T, Vp), dtype=torch.bfloat16, device=qx.q.device)
    stats = torch.empty((T, groups, 2), dtype=torch.float32, device=qx.q.device)
    gemm(operand(qx, C.K_MAJOR, d), operand(qw, C.MN_MAJOR, Vp), T, V, d, logits, Vp, epilogue=C.EPI_XENT,
         xent=(stats, groups, float(cap)))
    return logits, stats


def xent_combine(stats: torch.Tensor, logits: torch.Tensor, V: int, labels: torch.Tensor,
                 mask: torch.Tensor | None):
    """(lse, loss, qrow) from the XENT epilogue's partials (ufp8_xent_combine)."""
    T, groups = stats.shape[0], stats.shape[1]
    lse, loss, qrow = (torch.empty(T, dtype=torch.float32, device=logits.device) for _ in range(3))
    _launch("xent_combine", 8.0 * T * groups, lambda: C.xent_combine(
        stats.data_ptr(), groups, logits.data_ptr(), T, V, logits.stride(0), labels.data_ptr(),
        mask.data_ptr() if mask is not None else None, lse.data_ptr(), loss.data_ptr(), qrow.data_ptr(), _stream()))
    return lse, loss, qrow


def head_xent_forward(x2d: torch.Tensor, scale: torch.Tensor | None, centered: bool, eps: float, w: torch.Tensor,
                      labels: torch.Tensor, mask: torch.Tensor | None, cap: float):
    """Fused final norm -> FP8 lm_head -> next-token loss.  Returns (loss f32 [T], saved)."""
    x2d = _check_bf16_cuda(x2d, "x")
    V = w.shape[1]
    qx, rstd = rmsnorm_quant(x2d, scale, centered, eps, C.E4M3)
    qw = quantize_head_weight(w)
    logits, stats = head_logits(qx, qw, V, cap)
    lse, loss, qrow = xent_combine(stats, logits, V, labels, mask)
    return loss, (qx, rstd, qw, logits, lse, qrow, V)


def head_xent_backward(dloss: torch.Tensor, saved, labels: torch.Tensor, mask: torch.Tensor | None, cap: float,
                       need_dw: bool = True, fmt: int = C.E5M2):
    """Backward of head_xent_forward up to the norm: (dxn bf16 [T, d], dw bf16 [d, V] or None).
    `fmt`: the fp8 format of the logit gradient (the lm_head's bwd_dtype)."""
    qx, rstd, qw, logits, lse, qrow, V = saved
    T, d = qx.q.shape
    qd = xent_grad(logits, labels, mask, lse, qrow, dloss, cap, fmt, V)
    Vp = qd.q.shape[1]
    dxn = torch.empty((T, d), dtype=torch.bfloat16, device=qx.q.device)
    gemm(operand(qd, C.K_MAJOR, Vp), operand(qw, C.K_MAJOR, Vp), T, d, V, dxn, d)
    dw = None
    if need_dw:
        dw = torch.empty((d, V), dtype=torch.bfloat16, device=qx.q.device)
        gemm(operand(qx, C.MN_MAJOR, d), operand(qd, C.MN_MAJOR, Vp), d, V, T, dw, V)
    return dxn, dw


# ----------------------------------------------------------------------------- Newton-Schulz
def newton_schulz(g: torch.Tensor, coeffs, eps: float = 1e-8, out_dtype: torch.dtype | None = None) -> torch.Tensor:
    """ufp8_newton_schulz over g [batch, m, n] (f32 or bf16, CUDA): the orthogonalisation of Muon
    (ueaj/opt/multiscale.py:110-141) with one (a, b, c) triple per step.  Returns [batch, m, n] in
    out_dtype (default: g's dtype; f32 or bf16)."""
    if not g.is_cuda or g.dim() != 3 or g.dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("newton_schulz: expected a CUDA f32 or bf16 tensor [batch, m, n]")
    g = g.contiguous()
    batch, m, n = g.shape
    out_dtype = g.dtype if out_dtype is None else out_dtype
    out = torch.empty((batch, m, n), dtype=out_dtype, device=g.device)
    nbytes = C.newton_schulz_workspace(batch, m, n)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=g.device)
    dt = {torch.float32: C.OUT_F32, torch.bfloat16: C.OUT_BF16}
    s, l = min(m, n), max(m, n)
    # FLOPs executed: the symmetric X X^T and A A products compute only the tiles on or below
    # the diagonal (a 256-tile triangle), the update B X all of its product
    tiles = -(-s // 256)
    tri = (tiles * (tiles + 1) / 2) / (tiles * tiles)
    flops = float(batch) * len(coeffs) * (2.0 * s * s * l * (1.0 + tri) + 2.0 * s ** 3 * tri)
    _launch("newton_schulz", flops, lambda: C.newton_schulz(
        g.data_ptr(), dt[g.dtype], batch, m, n, coeffs, eps, out.data_ptr(), dt[out_dtype], ws.data_ptr(), nbytes,
        _stream()))
    return out
