"""Build recipe for libufp8.so (sm_100a only), in-tree at macrogpt_jax_b200/lib/.

Run as ``python -m macrogpt_jax_b200.build``.  nvcc cross-compiles for sm_100a without a GPU,
so the library is built on the development host and travels with the source tree.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB_PATH = LIB_DIR / "libufp8.so"
INCLUDE = PKG.parent / "include"
SOURCES = ["quant.cu", "norm.cu", "xent.cu", "ns.cu", "attn.cu", "gemm.cu", "tp.cu", "noalloc.cu", "capi.cu"]
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "ufp8.h"]
    return any(p.stat().st_mtime > built for p in deps if p.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles csrc/*.cu into lib/libufp8.so when a source is newer than the library."""
    if not force and not _stale():
        return LIB_PATH
    LIB_DIR.mkdir(exist_ok=True)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, *(["-Xptxas", "-v"] if verbose else []),
           "-o", str(tmp), *[str(CSRC / s) for s in SOURCES]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


XLA_LIB_PATH = LIB_DIR / "libufp8_xla.so"


def jax_ffi_include_dir() -> str | None:
    """jaxlib's XLA FFI header directory, or None when JAX is not installed."""
    try:
        import jax.ffi  # noqa: F401
        return jax.ffi.include_dir()
    except Exception:  # noqa: BLE001  (absent or too old a jax: no XLA binding)
        return None


def build_xla_ffi(force: bool = False) -> Path | None:
    """Compiles csrc/xla_ffi.cc (the XLA custom-call handlers) into lib/libufp8_xla.so, linked
    to libufp8.so, when jaxlib's headers are available; returns None (and builds nothing)
    otherwise.  The reference registers the handlers with jax.ffi.register_ffi_target."""
    inc = jax_ffi_include_dir()
    if inc is None:
        return None
    lib = build()
    src = CSRC / "xla_ffi.cc"
    if not force and XLA_LIB_PATH.exists() and XLA_LIB_PATH.stat().st_mtime > max(src.stat().st_mtime,
                                                                                   lib.stat().st_mtime):
        return XLA_LIB_PATH
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-I{inc}", f"-I{INCLUDE}", f"-I{cuda_home}/include",
           "-o", str(XLA_LIB_PATH), str(src), f"-L{LIB_DIR}", "-lufp8", "-Wl,-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed ({res.returncode}):\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
    return XLA_LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
    xla = build_xla_ffi(force="--force" in sys.argv)
    print(xla if xla is not None else "libufp8_xla.so skipped: jaxlib headers (jax.ffi.include_dir) not found")
