"""Shared helpers for the parity tests: numpy (oracle) <-> torch conversions and the
floating-point comparison used for GEMM outputs."""
from __future__ import annotations

import numpy as np
import torch

# Tolerance for bf16 GEMM outputs against the oracle (fp64 accumulate of the same fp8
# operands): max |D - R| <= REL_TOL * max |R|, and cosine similarity >= COS_TOL.
REL_TOL = 2e-2
COS_TOL = 0.9999


def bits_to_torch_bf16(bits: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(device)


def torch_bf16_to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def torch_fp8_to_codes(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy()


def bf16_bits_to_f64(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def compare(out: np.ndarray, ref: np.ndarray, rel_tol: float = REL_TOL, cos_tol: float = COS_TOL):
    """Returns (max_rel, cosine) and asserts both bounds.  Inputs are float arrays."""
    out = np.asarray(out, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    assert out.shape == ref.shape
    assert np.isfinite(out).all(), "non-finite values in the GPU output"
    scale = np.abs(ref).max()
    if scale == 0:
        assert np.abs(out).max() == 0
        return 0.0, 1.0
    max_rel = float(np.abs(out - ref).max() / scale)
    cos = float(out @ ref / (np.linalg.norm(out) * np.linalg.norm(ref)))
    assert max_rel <= rel_tol, f"max relative error {max_rel:.3e} > {rel_tol}"
    assert cos >= cos_tol, f"cosine {cos:.7f} < {cos_tol}"
    return max_rel, cos
