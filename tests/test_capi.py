"""libufp8.so on a machine without a GPU: it loads, exports every entry point include/ufp8.h
declares, and rejects bad requests on the host with an error code and message (no call
here reaches a kernel)."""
import ctypes
import re
from pathlib import Path

import pytest

from macrogpt_jax_b200 import _capi as C

HEADER = Path(__file__).resolve().parents[1] / "include" / "ufp8.h"


def _declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(ufp8_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_header_symbols():
    lib = C.load()
    declared = _declared()
    assert declared, "no declarations parsed from include/ufp8.h"
    for name in declared:
        assert hasattr(lib, name), f"{name} declared in ufp8.h but not exported"
    assert sorted(C.EXPORTED_SYMBOLS) == declared


def test_header_constants_match_binding():
    text = HEADER.read_text()
    consts = dict(re.findall(r"#define (UFP8_[A-Z0-9_]+) \(?(-?\d+)\)?", text))
    assert int(consts["UFP8_OK"]) == C.OK
    assert int(consts["UFP8_ERR_INVALID"]) == C.ERR_INVALID
    assert int(consts["UFP8_ERR_ALIGN"]) == C.ERR_ALIGN
    assert (int(consts["UFP8_E4M3"]), int(consts["UFP8_E5M2"])) == (C.E4M3, C.E5M2)
    assert (int(consts["UFP8_K_MAJOR"]), int(consts["UFP8_MN_MAJOR"])) == (C.K_MAJOR, C.MN_MAJOR)
    assert (int(consts["UFP8_EPI_STORE"]), int(consts["UFP8_EPI_SWIGLU"]), int(consts["UFP8_EPI_DSWIGLU"]),
            int(consts["UFP8_EPI_RS_PUSH"]), int(consts["UFP8_EPI_XENT"])) == \
        (C.EPI_STORE, C.EPI_SWIGLU, C.EPI_DSWIGLU, C.EPI_RS_PUSH, C.EPI_XENT)
    assert int(consts["UFP8_BF16"]) == C.BF16
    assert int(consts["UFP8_EPI_AXPBY"]) == C.EPI_AXPBY
    assert tuple(int(consts[k]) for k in ("UFP8_GEMM_AUTO", "UFP8_GEMM_SINGLE_CTA", "UFP8_GEMM_CTA_PAIR",
                                          "UFP8_GEMM_CTA_PAIR_DIRECT")) == \
        (C.GEMM_AUTO, C.GEMM_SINGLE_CTA, C.GEMM_CTA_PAIR, C.GEMM_CTA_PAIR_DIRECT)
    assert (int(consts["UFP8_STATUS_WAIT_TIMEOUT"]), int(consts["UFP8_STATUS_PEER_TIMEOUT"]),
            int(consts["UFP8_IPC_HANDLE_BYTES"])) == (C.STATUS_WAIT_TIMEOUT, C.STATUS_PEER_TIMEOUT, C.IPC_HANDLE_BYTES)
    assert int(consts["UFP8_ABI_VERSION"]) == C.load().ufp8_abi_version()


def test_struct_layout_matches_header(tmp_path):
    """Every field offset and struct size of the ctypes mirrors equals what the C compiler
    makes of include/ufp8.h."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    checks = [("ufp8_operand", C.Operand), ("ufp8_gemm_desc", C.GemmDesc), ("ufp8_attn_desc", C.AttnDesc)]
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "ufp8.h"', "int main(void) {"]
    for cname, py in checks:
        lines.append(f'printf("{cname} sizeof %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines.append("return 0; }")
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    include = Path(__file__).resolve().parents[1] / "include"
    subprocess.run([cc, "-I", str(include), str(src), "-o", str(exe)], check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        struct, field, value = line.split()
        got[(struct, field)] = int(value)
    for cname, py in checks:
        assert got[(cname, "sizeof")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)


@pytest.mark.parametrize("call,code,msg", [
    (lambda L: L.ufp8_gemm(None, None), C.ERR_INVALID, "null descriptor"),
    (lambda L: L.ufp8_rmsnorm_quant(None, 4, 0, 0, None, 0, 0, 1e-6, 0, None, None, None, None, None, 0, None),
     C.ERR_INVALID, "d > 0"),
    (lambda L: L.ufp8_rmsnorm_quant(None, 0, 8, 8, None, 0, 0, 1e-6, 0, None, None, None, None, None, 0, None),
     C.ERR_INVALID, "no output requested"),
    (lambda L: L.ufp8_rmsnorm_backward(None, 1, 8, 8, None, 0, 0, None, None, 8, None, 8, None, None, 0, None),
     C.ERR_INVALID, "null x"),
    (lambda L: L.ufp8_rmsnorm_backward(ctypes.c_void_p(16), 1, 9000, 9000, None, 0, 0, None, None, 9000, None, 9000,
                                       None, None, 0, None), C.ERR_UNSUPPORTED, "d 9000"),
    (lambda L: L.ufp8_xent_forward(None, 4, 0, 0, None, None, None, None, None, None), C.ERR_INVALID, "V >= 1"),
    (lambda L: L.ufp8_xent_forward(None, 2, 8, 4, None, None, None, None, None, None), C.ERR_INVALID, "ldl < V"),
    (lambda L: L.ufp8_xent_forward(None, 2, 8, 8, None, None, None, None, None, None), C.ERR_INVALID,
     "null logits"),
    (lambda L: L.ufp8_xent_combine(ctypes.c_void_p(16), 1, ctypes.c_void_p(16), 1, 300, 300, ctypes.c_void_p(16),
                                   None, None, None, None, None), C.ERR_INVALID, "ld_stats < ceil(V / 128)"),
    (lambda L: L.ufp8_xent_backward(ctypes.c_void_p(16), 1, 8, 8, ctypes.c_void_p(16), None, None, None, None, 0.0,
                                    5, None, 8, None, None, None), C.ERR_INVALID, "fmt 5"),
    (lambda L: L.ufp8_xent_backward(ctypes.c_void_p(16), 1, 8, 8, ctypes.c_void_p(16), None, None, None, None, -1.0,
                                    C.BF16, None, 8, None, None, None), C.ERR_INVALID, "cap must be"),
    (lambda L: L.ufp8_xent_backward(ctypes.c_void_p(16), 1, 8, 8, ctypes.c_void_p(16), None, None, None, None, 0.0,
                                    C.E5M2, ctypes.c_void_p(16), 8, None, None, None), C.ERR_INVALID,
     "null lse, qrow or dlogits"),
    (lambda L: L.ufp8_newton_schulz(None, 7, 1, 8, 8, 5, None, 1e-8, None, 0, None, 0, None), C.ERR_INVALID,
     "g_dtype"),
    (lambda L: L.ufp8_newton_schulz(None, C.OUT_F32, 1, 8, 8, 0, None, 1e-8, None, C.OUT_F32, None, 0, None),
     C.ERR_INVALID, "steps must be 1..64"),
    (lambda L: L.ufp8_newton_schulz(None, C.OUT_F32, 1, 12, 8, 1, (ctypes.c_float * 3)(1, 2, 3), 1e-8, None,
                                    C.OUT_F32, None, 0, None), C.ERR_UNSUPPORTED, "multiples of 8"),
    (lambda L: L.ufp8_newton_schulz(None, C.OUT_F32, 1, 16, 8, 1, (ctypes.c_float * 3)(1, 2, 3), 1e-8, None,
                                    C.OUT_F32, None, 0, None), C.ERR_INVALID, "workspace of"),
    (lambda L: L.ufp8_newton_schulz_workspace(-1, 8, 8, None), C.ERR_INVALID, "null pointer"),
    (lambda L: L.ufp8_amax(None, -1, None, None), C.ERR_INVALID, "n < 0"),
    (lambda L: L.ufp8_quantize(None, 4, 7, None, None, None, None), C.ERR_INVALID, "fmt 7"),
    (lambda L: L.ufp8_amax_quant(None, 4, 3, None, None, None, None), C.ERR_INVALID, "fmt 3"),
    (lambda L: L.ufp8_cast(None, -5, 0, None, None), C.ERR_INVALID, "n < 0"),
    (lambda L: L.ufp8_set_gemm_variant(9), C.ERR_INVALID, "unknown variant"),
    (lambda L: L.ufp8_set_gemm_ctas(-2), C.ERR_INVALID, "ctas < 0"),
    (lambda L: L.ufp8_device_status(None, 0), C.ERR_INVALID, "null pointer"),
])
def test_host_validation_errors(call, code, msg):
    lib = C.load()
    assert call(lib) == code
    assert msg in lib.ufp8_last_error().decode()


def test_python_wrapper_raises():
    with pytest.raises(C.UFP8Error) as e:
        C.set_gemm_variant(6)
    assert e.value.code == C.ERR_INVALID
    C.set_gemm_variant(0)


def test_ops_refuse_cpu_tensors():
    """There is no CPU path: the ops raise instead of computing on the host."""
    import torch
    from macrogpt_jax_b200 import ops
    with pytest.raises(ValueError, match="CUDA"):
        ops.quantize(torch.zeros(4, dtype=torch.bfloat16), C.E4M3)


def test_xla_ffi_shim_builds_when_jaxlib_is_present():
    """The XLA custom-call handlers (csrc/xla_ffi.cc) compile against jaxlib's headers and export
    every handler symbol; without JAX (as on these machines) the build is skipped, not failed."""
    from macrogpt_jax_b200 import build
    src = (build.CSRC / "xla_ffi.cc").read_text()
    handlers = sorted(re.findall(r"XLA_FFI_DEFINE_HANDLER_SYMBOL\((\w+),", src))
    assert handlers == ["Ufp8AmaxQuant", "Ufp8AmaxQuantNoalloc", "Ufp8AttentionBackward", "Ufp8AttentionForward",
                        "Ufp8Gemm", "Ufp8GmlpB2", "Ufp8GmlpF1", "Ufp8RmsnormQuant"]
    for entry in re.findall(r"\b(ufp8_[a-z0-9_]+)\(", src):
        assert hasattr(C.load(), entry), entry
    if build.jax_ffi_include_dir() is None:
        assert build.build_xla_ffi() is None
        pytest.skip("jaxlib headers not installed: the XLA FFI shim is not built here")
    lib = ctypes.CDLL(str(build.build_xla_ffi(force=True)))
    for h in handlers:
        assert hasattr(lib, h), h


def test_attention_workspace_sizes():
    """With the default positions the attention keeps S and dP out of memory: the forward
    workspace holds the per-row softmax partials (HI * n rows of ceil(n / 128) float2) and the
    backward one rowsum(dO O) plus dS; explicit positions take the materialised S / dP (f32).
    `saved` (P bf16 and lse of every batch element) is the same either way.  No device call."""
    al = lambda b: (b + 255) // 256 * 256  # noqa: E731
    b, n, H, I = 2, 520, 2, 4
    hi, nn, ld = H * I, n * n, (n + 127) // 128
    pos = (ctypes.c_int32 * 16)()  # any 16-byte aligned address stands for the position arrays
    fused = C.AttnDesc(b, n, H, I, 64, None, None, None, None, 0.125, 0)
    mat = C.AttnDesc(b, n, H, I, 64, None, None, ctypes.addressof(pos), ctypes.addressof(pos), 0.125, 0)
    f_fwd, f_saved, f_bwd = C.attention_workspace(fused)
    m_fwd, m_saved, m_bwd = C.attention_workspace(mat)
    saved = al(b * hi * nn * 2) + al(b * hi * n * 4)
    assert f_saved == m_saved == saved
    assert f_fwd == al(hi * n * ld * 8) and m_fwd == al(hi * nn * 4)
    assert f_bwd == al(hi * n * 4) + al(hi * nn * 2) and m_bwd == al(hi * nn * 4) + al(hi * nn * 2)
    with pytest.raises(C.UFP8Error, match="multiple of 8"):
        C.attention_workspace(C.AttnDesc(b, 522, H, I, 64, None, None, None, None, 0.125, 0))
