"""Generates the golden fixtures of the FP8 contraction path from the oracle (seed 0).

    python tests/golden/make_golden.py

Writes golden_v1.npz next to this script.  The reference's own program (JAX) cannot run on
these machines and the reference repository ships no test vectors for this path, so the
vectors come from the oracle, whose fp8 casts the tests pin against ml_dtypes 0.5.4 (the
reference's cast library).  Contents (bf16 as uint16 bit patterns, fp8 as uint8 codes):

  quant_{e4m3,e5m2}_{x,q,amax,inv}  per-tensor quantisation of 4099 N(0, 9) values with
                                    planted zeros, denormals, a max-bf16 and a NaN-free tail
  einsum_x, einsum_w, einsum_y      Einsum "bsd,df->bsf" forward in FP8 (B2, S8, D128, F256)
  gmlp_{x,wf,wd,dy}                 GMLP inputs (T 128, d 128, h 256)
  gmlp_{y,dx,dwf,dwd}               its FP8 forward output and gradients
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from oracle import fp8, path  # noqa: E402

OUT = Path(__file__).resolve().parent / "golden_v1.npz"


def build() -> dict:
    rng = np.random.default_rng(0)
    out = {}
    x = path.bf16_normal(rng, (4099,), 3.0)
    x[:7] = [0x0000, 0x8000, 0x0001, 0x8003, 0x7F7F, 0xFF7F, 0x3F80]  # zeros, denormals, +-max, 1.0
    for name, f in (("e4m3", fp8.E4M3), ("e5m2", fp8.E5M2)):
        q, a, inv = fp8.quantize_bits(x, f)
        out[f"quant_{name}_x"] = x
        out[f"quant_{name}_q"] = q
        out[f"quant_{name}_amax"] = np.array([a], np.float32)
        out[f"quant_{name}_inv"] = np.array([inv], np.float32)
    ex = path.bf16_normal(rng, (2, 8, 128))
    ew = path.bf16_normal(rng, (128, 256), 128 ** -0.5)
    ey, _, _ = path.einsum_fp8("bsd,df->bsf", ex, ew)
    out.update(einsum_x=ex, einsum_w=ew, einsum_y=ey)
    T, d, h = 128, 128, 256
    gx = path.bf16_normal(rng, (T, d))
    gwf = path.bf16_normal(rng, (2, d, h), d ** -0.5)
    gwd = path.bf16_normal(rng, (h, d), h ** -0.5)
    gdy = path.bf16_normal(rng, (T, d), 1e-3)
    y, saved = path.gmlp_forward(gx, gwf, gwd)
    g = path.gmlp_backward(gdy, saved)
    out.update(gmlp_x=gx, gmlp_wf=gwf, gmlp_wd=gwd, gmlp_dy=gdy, gmlp_y=y, gmlp_dx=g["dx"], gmlp_dwf=g["dwf"],
               gmlp_dwd=g["dwd"])
    return out


if __name__ == "__main__":
    np.savez_compressed(OUT, **build())
    print(OUT)
