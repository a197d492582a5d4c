"""Per-kernel micro-benchmark of the GMLP contractions (CUDA-event timing, one GPU).

    python -m macrogpt_jax_b200.kernel_bench [--tokens T] [--d D] [--hidden H]
                                             [--gemms F1,F2,B2,B1,B4,B3] [--reps R] [--warmup W]

Each named GEMM of the GMLP step runs R times after W warm-up launches on seeded fp8
operands; the script prints one line per GEMM with its mean duration and TFLOP/s.  With
--reps 1 --warmup 1 it doubles as a small, self-contained target for profilers.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import _capi as C
from . import ops

ALL = ("F1", "F2", "B2", "B1", "B4", "B3")


def _fp8(shape, fmt, dev, gen, std=1.0):
    x = (torch.randn(shape, generator=gen, device=dev) * std).to(torch.bfloat16)
    return ops.quantize(x, fmt)


def build(T, d, h, dev):
    """Operands and outputs of the six GMLP GEMMs; returns {name: (flops, launch_fn)}."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    qx = _fp8((T, d), C.E4M3, dev, gen)
    qwf = _fp8((2, d, h), C.E4M3, dev, gen, d ** -0.5)
    qwd = _fp8((h, d), C.E4M3, dev, gen, h ** -0.5)
    qh = _fp8((T, h), C.E4M3, dev, gen)
    qdy = _fp8((T, d), C.E5M2, dev, gen, 1e-3)
    qdug = _fp8((2, T, h), C.E5M2, dev, gen, 1e-3)
    ug = torch.randn((2, T, h), generator=gen, device=dev).to(torch.bfloat16)
    g = {
        "F1": (4.0 * T * d * h, lambda: ops.gmlp_f1(qx, qwf)),
        "F2": (2.0 * T * d * h, lambda: ops.gmlp_f2(qh, qwd)),
        "B2": (2.0 * T * d * h, lambda: ops.gmlp_b2(qdy, qwd, ug)),
        "B1": (2.0 * T * d * h, lambda: ops.gmlp_b1(qh, qdy)),
        "B4": (4.0 * T * d * h, lambda: ops.gmlp_b4(qdug, qwf)),
        "B3": (4.0 * T * d * h, lambda: ops.gmlp_b3(qx, qdug)),
    }
    return g


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=14336)
    ap.add_argument("--gemms", default=",".join(ALL))
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--variant", type=int, default=0, help="0 auto, 1 one CTA per tile, 2 CTA pair")
    args = ap.parse_args()
    C.set_gemm_variant(args.variant)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = build(args.tokens, args.d, args.hidden, dev)
    names = [n.strip() for n in args.gemms.split(",") if n.strip()]
    for n in names:
        if n not in g:
            raise SystemExit(f"unknown GEMM {n}; choose from {ALL}")
    for n in names:  # warm-up, in order
        for _ in range(args.warmup):
            g[n][1]()
    torch.cuda.synchronize()
    for n in names:
        flops, fn = g[n]
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.reps):
            fn()
        e.record()
        torch.cuda.synchronize()
        us = s.elapsed_time(e) * 1000.0 / args.reps
        print(json.dumps({"gemm": n, "variant": args.variant, "tokens": args.tokens, "d": args.d, "hidden": args.hidden, "us": us,
                          "tflops": flops / us / 1e6}), flush=True)
    if C.device_status() != 0:
        raise SystemExit("device status word set: a kernel wait timed out")


if __name__ == "__main__":
    main()
