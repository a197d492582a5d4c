"""ctypes binding of libufp8.so (the C ABI declared in include/ufp8.h).

There is no fallback: if the library is missing or cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libufp8.so"

# Constants mirrored from include/ufp8.h.
OK = 0
ERR_INVALID, ERR_ALIGN, ERR_UNSUPPORTED, ERR_CUDA, ERR_DEVICE = -1, -2, -3, -4, -5
STATUS_WAIT_TIMEOUT, STATUS_PEER_TIMEOUT = 1, 2
IPC_HANDLE_BYTES = 64
AG_COPY_ENGINE, AG_SM = 0, 1
E4M3, E5M2 = 0, 1
BF16 = 2  # bf16 GEMM operands; unquantised output of ufp8_xent_backward
K_MAJOR, MN_MAJOR = 0, 1
OUT_BF16, OUT_F32 = 0, 1
EPI_STORE, EPI_SWIGLU, EPI_DSWIGLU, EPI_RS_PUSH, EPI_XENT, EPI_AXPBY = 0, 1, 2, 3, 4, 5
EPI_ATTN_STATS, EPI_ATTN_P, EPI_ATTN_DS = 6, 7, 8
TILES_ALL, TILES_LOWER, TILES_K_TO_DIAG, TILES_K_FROM_DIAG = 0, 1, 2, 3
GEMM_AUTO, GEMM_SINGLE_CTA, GEMM_CTA_PAIR, GEMM_CTA_PAIR_DIRECT, GEMM_CTA_PAIR_WIDE, GEMM_CTA_PAIR_N512 = (
    0, 1, 2, 3, 4, 5)

EXPORTED_SYMBOLS = (
    "ufp8_last_error",
    "ufp8_abi_version",
    "ufp8_amax",
    "ufp8_quantize",
    "ufp8_amax_quant",
    "ufp8_cast",
    "ufp8_gemm",
    "ufp8_device_status",
    "ufp8_set_gemm_ctas",
    "ufp8_set_gemm_variant",
    "ufp8_set_gemm_raster",
    "ufp8_tp_create",
    "ufp8_tp_connect",
    "ufp8_tp_connect_local",
    "ufp8_tp_destroy",
    "ufp8_tp_set_timeout_ms",
    "ufp8_tp_slot_bytes",
    "ufp8_tp_begin",
    "ufp8_tp_finish",
    "ufp8_tp_allreduce_max",
    "ufp8_tp_local",
    "ufp8_tp_ag_push",
    "ufp8_tp_set_copy_lanes",
    "ufp8_tp_rs_push_copy",
    "ufp8_amax_quant_noalloc",
    "ufp8_rmsnorm_quant",
    "ufp8_rmsnorm_backward_workspace",
    "ufp8_rmsnorm_backward",
    "ufp8_xent_forward",
    "ufp8_xent_combine",
    "ufp8_xent_backward",
    "ufp8_newton_schulz_workspace",
    "ufp8_newton_schulz",
    "ufp8_rope_table",
    "ufp8_rope",
    "ufp8_attention_workspace",
    "ufp8_attention_forward",
    "ufp8_attention_backward",
)


class Operand(ctypes.Structure):
    _fields_ = [
        ("ptr", ctypes.c_void_p),
        ("fmt", ctypes.c_int32),
        ("major", ctypes.c_int32),
        ("ld", ctypes.c_int64),
        ("batch_stride", ctypes.c_int64),
        ("batch_count", ctypes.c_int32),
        ("batch_group", ctypes.c_int32),
        ("inv_scale", ctypes.c_void_p),
    ]


class GemmDesc(ctypes.Structure):
    _fields_ = [
        ("M", ctypes.c_int64),
        ("N", ctypes.c_int64),
        ("K", ctypes.c_int64),
        ("batch", ctypes.c_int32),
        ("k_batches", ctypes.c_int32),
        ("a", Operand),
        ("b", Operand),
        ("d", ctypes.c_void_p),
        ("d_dtype", ctypes.c_int32),
        ("epilogue", ctypes.c_int32),
        ("ldd", ctypes.c_int64),
        ("d_batch_stride", ctypes.c_int64),
        ("h", ctypes.c_void_p),
        ("ldh", ctypes.c_int64),
        ("ug", ctypes.c_void_p),
        ("ldug", ctypes.c_int64),
        ("ug_batch_stride", ctypes.c_int64),
        ("amax_out", ctypes.c_void_p),
        ("rs_slots", ctypes.c_void_p),
        ("rs_rank", ctypes.c_int32),
        ("rs_reserved", ctypes.c_int32),
        ("rs_rows_per_rank", ctypes.c_int64),
        ("ag_flags", ctypes.c_void_p),
        ("ag_epoch", ctypes.c_uint32),
        ("ag_rank", ctypes.c_int32),
        ("ag_rows_per_rank", ctypes.c_int64),
        ("xent_stats", ctypes.c_void_p),
        ("xent_ld_stats", ctypes.c_int64),
        ("xent_cap", ctypes.c_float),
        ("xent_reserved", ctypes.c_int32),
        ("c", ctypes.c_void_p),
        ("ldc", ctypes.c_int64),
        ("c_batch_stride", ctypes.c_int64),
        ("alpha", ctypes.c_float),
        ("beta", ctypes.c_float),
        ("tile_mask", ctypes.c_int32),
        ("reserved2", ctypes.c_int32),
        ("attn_q_segment_ids", ctypes.c_void_p),
        ("attn_kv_segment_ids", ctypes.c_void_p),
        ("attn_stats", ctypes.c_void_p),
        ("attn_ld_stats", ctypes.c_int64),
        ("attn_row", ctypes.c_void_p),
        ("attn_scale", ctypes.c_float),
        ("attn_reserved", ctypes.c_int32),
    ]


class AttnDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64),
        ("seq", ctypes.c_int64),
        ("kv_heads", ctypes.c_int64),
        ("group", ctypes.c_int64),
        ("head_dim", ctypes.c_int64),
        ("q_segment_ids", ctypes.c_void_p),
        ("kv_segment_ids", ctypes.c_void_p),
        ("q_positions", ctypes.c_void_p),
        ("kv_positions", ctypes.c_void_p),
        ("scale", ctypes.c_float),
        ("reserved", ctypes.c_int32),
    ]


class UFP8Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"ufp8 error {code}: {msg}")
        self.code = code


_lib = None

# Number of kernels this library has launched from this process (host-side count).
launches = 0


def load() -> ctypes.CDLL:
    """Loads libufp8.so once; raises if it is absent (no fallback path exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"libufp8.so not built at {LIB_PATH}; run `python -m macrogpt_jax_b200.build`")
    lib = ctypes.CDLL(str(LIB_PATH))
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.ufp8_last_error.restype = ctypes.c_char_p
    lib.ufp8_last_error.argtypes = []
    lib.ufp8_abi_version.restype = i32
    lib.ufp8_amax.argtypes = [vp, i64, vp, vp]
    lib.ufp8_quantize.argtypes = [vp, i64, i32, vp, vp, vp, vp]
    lib.ufp8_amax_quant.argtypes = [vp, i64, i32, vp, vp, vp, vp]
    lib.ufp8_cast.argtypes = [vp, i64, i32, vp, vp]
    lib.ufp8_amax_quant_noalloc.argtypes = [vp, i64, i32, vp, vp, vp]
    lib.ufp8_gemm.argtypes = [ctypes.POINTER(GemmDesc), vp]
    lib.ufp8_device_status.argtypes = [ctypes.POINTER(ctypes.c_int), i32]
    lib.ufp8_set_gemm_ctas.argtypes = [i32]
    lib.ufp8_set_gemm_variant.argtypes = [i32]
    lib.ufp8_set_gemm_raster.argtypes = [i32]
    lib.ufp8_tp_create.argtypes = [i32, i32, i64, ctypes.POINTER(vp), ctypes.c_char_p]
    lib.ufp8_tp_connect.argtypes = [vp, ctypes.c_char_p]
    lib.ufp8_tp_connect_local.argtypes = [vp, ctypes.POINTER(vp)]
    lib.ufp8_tp_destroy.argtypes = [vp]
    lib.ufp8_tp_set_timeout_ms.argtypes = [vp, i32]
    lib.ufp8_tp_slot_bytes.argtypes = [vp, ctypes.POINTER(i64)]
    lib.ufp8_tp_begin.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_uint64)]
    lib.ufp8_tp_finish.argtypes = [vp, ctypes.c_uint64, i64, i64, i64, vp, i64, vp]
    lib.ufp8_tp_allreduce_max.argtypes = [vp, vp, vp, i32, vp]
    lib.ufp8_tp_local.argtypes = [vp, ctypes.c_uint64, ctypes.POINTER(vp), ctypes.POINTER(vp)]
    lib.ufp8_tp_ag_push.argtypes = [vp, ctypes.c_uint64, i64, i32, vp]
    lib.ufp8_tp_set_copy_lanes.argtypes = [vp, i32]
    lib.ufp8_tp_rs_push_copy.argtypes = [vp, ctypes.c_uint64, vp, i64, i64, i64, vp]
    f32 = ctypes.c_float
    lib.ufp8_rmsnorm_quant.argtypes = [vp, i64, i64, i64, vp, i64, i32, f32, i32, vp, vp, vp, vp, vp, i64, vp]
    lib.ufp8_rmsnorm_backward_workspace.argtypes = [i64, i64, ctypes.POINTER(i64)]
    lib.ufp8_rmsnorm_backward.argtypes = [vp, i64, i64, i64, vp, i64, i32, vp, vp, i64, vp, i64, vp, vp, i64, vp]
    lib.ufp8_xent_forward.argtypes = [vp, i64, i64, i64, vp, vp, vp, vp, vp, vp]
    lib.ufp8_xent_combine.argtypes = [vp, i64, vp, i64, i64, i64, vp, vp, vp, vp, vp, vp]
    lib.ufp8_xent_backward.argtypes = [vp, i64, i64, i64, vp, vp, vp, vp, vp, f32, i32, vp, i64, vp, vp, vp]
    lib.ufp8_newton_schulz_workspace.argtypes = [i64, i64, i64, ctypes.POINTER(i64)]
    lib.ufp8_newton_schulz.argtypes = [vp, i32, i64, i64, i64, i32, vp, f32, vp, i32, vp, i64, vp]
    lib.ufp8_rope_table.argtypes = [vp, i64, i64, vp, vp, vp, vp]
    lib.ufp8_rope.argtypes = [vp, i64, i64, i64, vp, vp, i64, i32, vp, vp]
    ap = ctypes.POINTER(AttnDesc)
    lib.ufp8_attention_workspace.argtypes = [ap, ctypes.POINTER(i64), ctypes.POINTER(i64), ctypes.POINTER(i64)]
    lib.ufp8_attention_forward.argtypes = [ap, vp, vp, vp, vp, vp, vp, vp]
    lib.ufp8_attention_backward.argtypes = [ap, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]
    for name in ("ufp8_amax", "ufp8_quantize", "ufp8_amax_quant", "ufp8_cast", "ufp8_gemm", "ufp8_device_status",
                 "ufp8_set_gemm_ctas", "ufp8_set_gemm_variant", "ufp8_set_gemm_raster", "ufp8_tp_create",
                 "ufp8_tp_connect", "ufp8_tp_connect_local", "ufp8_tp_destroy", "ufp8_tp_set_timeout_ms", "ufp8_tp_slot_bytes", "ufp8_tp_begin",
                 "ufp8_tp_finish", "ufp8_tp_allreduce_max", "ufp8_amax_quant_noalloc",
                 "ufp8_tp_local", "ufp8_tp_ag_push", "ufp8_tp_set_copy_lanes", "ufp8_tp_rs_push_copy",
                 "ufp8_rmsnorm_quant", "ufp8_rmsnorm_backward_workspace",
                 "ufp8_rmsnorm_backward", "ufp8_xent_forward", "ufp8_xent_combine", "ufp8_xent_backward",
                 "ufp8_newton_schulz_workspace", "ufp8_newton_schulz", "ufp8_rope_table", "ufp8_rope",
                 "ufp8_attention_workspace", "ufp8_attention_forward", "ufp8_attention_backward"):
        getattr(lib, name).restype = i32
    _lib = lib
    return lib


def check(rc: int) -> None:
    if rc != OK:
        raise UFP8Error(rc, load().ufp8_last_error().decode(errors="replace"))


def _count(k: int) -> None:
    global launches
    launches += k


def amax(x_ptr: int, n: int, amax_ptr: int, stream: int) -> None:
    check(load().ufp8_amax(x_ptr, n, amax_ptr, stream))
    _count(1 if n > 0 else 0)


def quantize(x_ptr: int, n: int, fmt: int, amax_ptr: int, q_ptr: int, inv_ptr: int, stream: int) -> None:
    check(load().ufp8_quantize(x_ptr, n, fmt, amax_ptr, q_ptr, inv_ptr, stream))
    _count(1)


def amax_quant(x_ptr: int, n: int, fmt: int, q_ptr: int, amax_ptr: int, inv_ptr: int, stream: int) -> None:
    check(load().ufp8_amax_quant(x_ptr, n, fmt, q_ptr, amax_ptr, inv_ptr, stream))
    _count(2 if n > 0 else 1)


def amax_quant_noalloc(x_ptr: int, n: int, fmt: int, q_ptr: int, inv_ptr: int, stream: int) -> None:
    """ufp8_amax_quant with the amax scratch in the library's static device arrays."""
    check(load().ufp8_amax_quant_noalloc(x_ptr, n, fmt, q_ptr, inv_ptr, stream))
    _count(3 if n > 0 else 2)


def cast(x_ptr: int, n: int, fmt: int, q_ptr: int, stream: int) -> None:
    check(load().ufp8_cast(x_ptr, n, fmt, q_ptr, stream))
    _count(1 if n > 0 else 0)


def rmsnorm_quant(x_ptr, rows, d, ldx, scale_ptr, scale_len, centered, eps, fmt, q_ptr, amax_ptr, inv_ptr,
                  rstd_ptr, y_ptr, ldy, stream) -> None:
    """ufp8_rmsnorm_quant: RMSNorm rows of x (rstd out), optional bf16 y, optional fp8 q."""
    check(load().ufp8_rmsnorm_quant(x_ptr, rows, d, ldx, scale_ptr, scale_len, 1 if centered else 0, eps, fmt,
                                    q_ptr, amax_ptr, inv_ptr, rstd_ptr, y_ptr, ldy, stream))
    _count((1 if rows > 0 else 0) + (1 if inv_ptr else 0))


def rmsnorm_backward_workspace(rows: int, d: int) -> int:
    out = ctypes.c_int64(0)
    check(load().ufp8_rmsnorm_backward_workspace(rows, d, ctypes.byref(out)))
    return out.value


def rmsnorm_backward(x_ptr, rows, d, ldx, scale_ptr, scale_len, centered, rstd_ptr, dy_ptr, lddy, dx_ptr, lddx,
                     dscale_ptr, ws_ptr, ws_bytes, stream) -> None:
    check(load().ufp8_rmsnorm_backward(x_ptr, rows, d, ldx, scale_ptr, scale_len, 1 if centered else 0, rstd_ptr,
                                       dy_ptr, lddy, dx_ptr, lddx, dscale_ptr, ws_ptr, ws_bytes, stream))
    _count((1 if (rows > 0 or dscale_ptr) else 0) + (1 if dscale_ptr else 0))


def xent_forward(logits_ptr, rows, V, ldl, labels_ptr, mask_ptr, lse_ptr, loss_ptr, qrow_ptr, stream) -> None:
    """ufp8_xent_forward: per-row lse, masked loss and qrow from bf16 logits."""
    check(load().ufp8_xent_forward(logits_ptr, rows, V, ldl, labels_ptr, mask_ptr, lse_ptr, loss_ptr, qrow_ptr,
                                   stream))
    _count(1 if rows > 0 else 0)


def xent_combine(stats_ptr, ld_stats, logits_ptr, rows, V, ldl, labels_ptr, mask_ptr, lse_ptr, loss_ptr, qrow_ptr,
                 stream) -> None:
    """ufp8_xent_combine: the per-row results from the partials of a UFP8_EPI_XENT GEMM."""
    check(load().ufp8_xent_combine(stats_ptr, ld_stats, logits_ptr, rows, V, ldl, labels_ptr, mask_ptr, lse_ptr,
                                   loss_ptr, qrow_ptr, stream))
    _count(1 if rows > 0 else 0)


def xent_backward(logits_ptr, rows, V, ldl, labels_ptr, mask_ptr, lse_ptr, qrow_ptr, dloss_ptr, cap, fmt, out_ptr,
                  ldo, amax_ptr, inv_ptr, stream) -> None:
    """ufp8_xent_backward: dlogits (fp8 with its per-tensor scale, or bf16)."""
    check(load().ufp8_xent_backward(logits_ptr, rows, V, ldl, labels_ptr, mask_ptr, lse_ptr, qrow_ptr, dloss_ptr,
                                    cap, fmt, out_ptr, ldo, amax_ptr, inv_ptr, stream))
    _count((1 if fmt != BF16 else 0) + (1 if rows > 0 else 0))


def newton_schulz_workspace(batch: int, m: int, n: int) -> int:
    out = ctypes.c_int64(0)
    check(load().ufp8_newton_schulz_workspace(batch, m, n, ctypes.byref(out)))
    return out.value


def newton_schulz(g_ptr, g_dtype, batch, m, n, coeffs, eps, out_ptr, out_dtype, ws_ptr, ws_bytes, stream) -> None:
    """ufp8_newton_schulz; coeffs: a sequence of (a, b, c) triples, one per step."""
    flat = [float(v) for abc in coeffs for v in abc]
    arr = (ctypes.c_float * len(flat))(*flat)
    check(load().ufp8_newton_schulz(g_ptr, g_dtype, batch, m, n, len(flat) // 3, arr, eps, out_ptr, out_dtype,
                                    ws_ptr, ws_bytes, stream))
    _count((2 + 3 * (len(flat) // 3)) if batch > 0 else 0)


def rope_table(pos_ptr, count, half, inv_freq_ptr, sin_ptr, cos_ptr, stream) -> None:
    check(load().ufp8_rope_table(pos_ptr, count, half, inv_freq_ptr, sin_ptr, cos_ptr, stream))
    _count(1 if count > 0 else 0)


def rope(x_ptr, tokens, heads, d, sin_ptr, cos_ptr, period, inverse, out_ptr, stream) -> None:
    check(load().ufp8_rope(x_ptr, tokens, heads, d, sin_ptr, cos_ptr, period, 1 if inverse else 0, out_ptr, stream))
    _count(1 if tokens > 0 else 0)


def attention_workspace(desc: AttnDesc):
    """(forward workspace, saved, backward workspace) bytes."""
    f, s, b = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int64(0)
    check(load().ufp8_attention_workspace(ctypes.byref(desc), ctypes.byref(f), ctypes.byref(s), ctypes.byref(b)))
    return f.value, s.value, b.value


def attention_forward(desc: AttnDesc, q, k, v, out, saved, ws, stream) -> None:
    check(load().ufp8_attention_forward(ctypes.byref(desc), q, k, v, out, saved, ws, stream))
    _count(desc.batch * (2 * desc.kv_heads + 1))


def attention_backward(desc: AttnDesc, q, k, v, out, dout, saved, dq, dk, dv, ws, stream) -> None:
    check(load().ufp8_attention_backward(ctypes.byref(desc), q, k, v, out, dout, saved, dq, dk, dv, ws, stream))
    _count(desc.batch * (4 * desc.kv_heads + 1))


def gemm(desc: GemmDesc, stream: int) -> None:
    check(load().ufp8_gemm(ctypes.byref(desc), stream))
    _count(1 if desc.M > 0 and desc.N > 0 else 0)


def device_status(clear: bool = True) -> int:
    out = ctypes.c_int(0)
    check(load().ufp8_device_status(ctypes.byref(out), 1 if clear else 0))
    return out.value


def set_gemm_ctas(ctas: int) -> None:
    check(load().ufp8_set_gemm_ctas(ctas))


def set_gemm_variant(variant: int) -> None:
    check(load().ufp8_set_gemm_variant(variant))


def set_gemm_raster(group_m: int) -> None:
    check(load().ufp8_set_gemm_raster(group_m))


class TPReduceScatter:
    """One tensor-parallel context (include/ufp8.h ufp8_tp_*): peer-mapped staging slots of
    `slot_bytes` per source rank, double-buffered; serves reduce-scatters (RS_PUSH + finish),
    all-gathers (ag_push) and small MAX all-reduces."""

    def __init__(self, rank: int, world: int, slot_bytes: int):
        self.ctx = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
        check(load().ufp8_tp_create(rank, world, slot_bytes, ctypes.byref(self.ctx), handle))
        self.handle = handle.raw
        self.rank, self.world, self.slot_bytes = rank, world, slot_bytes
        self.epoch = 0  # last epoch begun

    def connect(self, handles) -> None:
        check(load().ufp8_tp_connect(self.ctx, b"".join(handles)))

    def connect_local(self, contexts) -> None:
        """Peers in this process: contexts[r] is the TPReduceScatter of rank r."""
        arr = (ctypes.c_void_p * len(contexts))(*[c.ctx.value for c in contexts])
        check(load().ufp8_tp_connect_local(self.ctx, arr))

    def set_timeout_ms(self, ms: int) -> None:
        check(load().ufp8_tp_set_timeout_ms(self.ctx, ms))

    def begin(self):
        """-> (device address of this epoch's slot table, epoch)"""
        table = ctypes.c_void_p()
        epoch = ctypes.c_uint64()
        check(load().ufp8_tp_begin(self.ctx, ctypes.byref(table), ctypes.byref(epoch)))
        self.epoch = epoch.value
        return table.value, epoch.value

    def finish(self, epoch: int, rows: int, cols: int, ld_slot: int, out_ptr: int, ld_out: int, stream: int) -> None:
        check(load().ufp8_tp_finish(self.ctx, epoch, rows, cols, ld_slot, out_ptr, ld_out, stream))
        _count(1)

    def local(self, epoch: int):
        """(data pointer, flags pointer) of this rank's buffer of `epoch`."""
        data, flags = ctypes.c_void_p(), ctypes.c_void_p()
        check(load().ufp8_tp_local(self.ctx, epoch, ctypes.byref(data), ctypes.byref(flags)))
        return data.value, flags.value

    def ag_push(self, epoch: int, nbytes: int, stream: int, engine: int = AG_COPY_ENGINE) -> None:
        """Copies this rank's slot of `epoch`'s buffer into every peer's (AG_SM: a small kernel;
        AG_COPY_ENGINE: copy engines), each followed by the arrival flag."""
        check(load().ufp8_tp_ag_push(self.ctx, epoch, nbytes, engine, stream))
        _count(1 if engine == AG_SM and self.world > 1 else 0)

    def set_copy_lanes(self, lanes: int) -> None:
        """Streams (1..8) over which the copy-engine pushes spread their per-peer copies."""
        check(load().ufp8_tp_set_copy_lanes(self.ctx, lanes))

    def rs_push_copy(self, epoch: int, src_ptr: int, ld_src: int, rows: int, cols: int, stream: int) -> None:
        """Copy-engine reduce-scatter push: block p of the k * rows partial rows (bf16, pitch
        ld_src) into slot [rank] of rank p's buffer of `epoch`; finish with ld_slot = cols."""
        check(load().ufp8_tp_rs_push_copy(self.ctx, epoch, src_ptr, ld_src, rows, cols, stream))

    def allreduce_max(self, in_ptr: int, out_ptr: int, n: int, stream: int) -> None:
        """Elementwise MAX over the group of n (1..8) non-negative device f32 values."""
        check(load().ufp8_tp_allreduce_max(self.ctx, in_ptr, out_ptr, n, stream))
        _count(1)

    def close(self) -> None:
        if self.ctx:
            load().ufp8_tp_destroy(self.ctx)
            self.ctx = ctypes.c_void_p()
