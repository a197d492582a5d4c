"""Per-kernel micro-benchmark of the GMLP contractions (CUDA-event timing, one GPU).

    python -m macrogpt_jax_b200.kernel_bench [--tokens T] [--d D] [--hidden H]
                                             [--gemms F1,F2,B2,B1,B4,B3] [--reps R] [--warmup W]
                                             [--variant V] [--seconds S] [--cublas]
                                             [--quant | --norm | --rs-push | --xent | --ns |
                                              --attn [--batch B --seq S --kv-heads H --group I]]

Each named GEMM of the GMLP step runs R times after W warm-up launches on seeded fp8
operands; the script prints one line per GEMM with its mean duration and TFLOP/s.  With
--reps 1 --warmup 1 it doubles as a small, self-contained target for profilers.  With
--seconds S each GEMM instead loops for S seconds while nvidia-smi samples the SM clock and
power (sustained, power-capped throughput).  --cublas adds the same-shape plain fp8 GEMM
from cuBLAS (torch._scaled_mm, per-tensor scales, bf16 out) as a library reference point.
"""
from __future__ import annotations

import argparse
import json
import statistics
import subprocess
import time

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


def cublas_same_shapes(T, d, h, dev):
    """Plain fp8 GEMMs of the GMLP shapes via cuBLAS (torch._scaled_mm), K-major operands."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    one = torch.ones((), device=dev)
    out = {}
    for name, (M, N, K) in {"F1": (T, 2 * h, d), "F2": (T, d, h), "B4": (T, d, 2 * h)}.items():
        a = torch.randn((M, K), generator=gen, device=dev).to(torch.float8_e4m3fn)
        b = (torch.randn((N, K), generator=gen, device=dev) * 0.05).to(torch.float8_e4m3fn)
        out["cublas_" + name] = (2.0 * M * N * K, lambda a=a, b=b: torch._scaled_mm(
            a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16))
    return out


def sustained(fn, seconds: float, gpu: int):
    """Loops fn for `seconds`; returns (mean ms per call, median SM MHz, max W, samples)."""
    smi = None
    try:
        smi = subprocess.Popen(["nvidia-smi", f"--id={gpu}", "--query-gpu=clocks.sm,power.draw",
                                "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE, text=True)
    except (OSError, FileNotFoundError):
        smi = None
    time.sleep(0.3)
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n, t0 = 0, time.time()
    s.record()
    while time.time() - t0 < seconds:
        fn()
        n += 1
        if n % 16 == 0:
            torch.cuda.synchronize()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / n
    mhz = power = None
    samples = 0
    if smi is not None:
        smi.terminate()
        rows = [r.split(", ") for r in smi.communicate()[0].strip().splitlines() if r.strip()]
        rows = rows[4:-2] if len(rows) > 8 else rows
        samples = len(rows)
        if rows:
            mhz = statistics.median(float(r[0]) for r in rows)
            power = max(float(r[1]) for r in rows)
    return ms, mhz, power, samples


def _time_us(fn, reps: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    s.record()
    for _ in range(reps):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) * 1000.0 / reps


def rs_push_bench(args, dev):
    """The down-projection (F2) and dx (B4) GEMMs of a TP-k GMLP shard (hidden h/k) on GPU 0,
    storing locally vs pushing every row into its owner's reduce-scatter slot (RS_PUSH) with
    owner 0 on GPU 0 and owners 1..k-1 on GPU 1 through a peer mapping; checks the pushed rows
    bit for bit and prints the achieved remote bytes per second.  Needs 2 GPUs with peer access."""
    if torch.cuda.device_count() < 2 or not torch.cuda.can_device_access_peer(0, 1):
        raise SystemExit("--rs-push needs two GPUs with peer access")
    from cuda.bindings import runtime as rt
    err = rt.cudaDeviceEnablePeerAccess(1, 0)[0]
    if err not in (rt.cudaError_t.cudaSuccess, rt.cudaError_t.cudaErrorPeerAccessAlreadyEnabled):
        raise SystemExit(f"cudaDeviceEnablePeerAccess: {err}")
    T, d = args.tokens, args.d
    peer = torch.device("cuda", 1)
    for world in (2, 4, 8):
        hl = args.hidden // world
        gen = torch.Generator(device=dev)
        gen.manual_seed(3)
        qh = _fp8((T, hl), C.E4M3, dev, gen)
        qwd = _fp8((hl, d), C.E4M3, dev, gen, hl ** -0.5)
        qdug = _fp8((2, T, hl), C.E5M2, dev, gen, 1e-3)
        qwf = _fp8((2, d, hl), C.E4M3, dev, gen, d ** -0.5)
        rl = T // world
        own = torch.empty((rl * world, d), dtype=torch.bfloat16, device=dev)
        remote = torch.zeros((world, rl * world, d), dtype=torch.bfloat16, device=peer)
        torch.cuda.synchronize(peer)
        table = torch.tensor([own.data_ptr()] + [remote[o].data_ptr() for o in range(1, world)],
                             dtype=torch.int64, device=dev)
        y_ref = ops.gmlp_f2(qh, qwd)
        ops.gmlp_f2_push(qh, qwd, table.data_ptr(), 0, rl)
        torch.cuda.synchronize()
        exact = torch.equal(own[:rl], y_ref[:rl]) and all(
            torch.equal(remote[o][:rl].cpu(), y_ref[o * rl:(o + 1) * rl].cpu()) for o in range(1, world))
        remote_bytes = T * d * 2 * (world - 1) / world
        rec = {"mode": "rs_push", "tp": world, "tokens": T, "d": d, "hidden_local": hl, "pushed_rows_exact": exact}
        for name, flops, local_fn, push_fn in (
                ("F2", 2.0 * T * d * hl, lambda: ops.gmlp_f2(qh, qwd),
                 lambda: ops.gmlp_f2_push(qh, qwd, table.data_ptr(), 0, rl)),
                ("B4", 4.0 * T * d * hl, lambda: ops.gmlp_b4(qdug, qwf),
                 lambda: ops.gmlp_b4_push(qdug, qwf, table.data_ptr(), 0, rl))):
            t_local = _time_us(local_fn, args.reps, args.warmup)
            t_push = _time_us(push_fn, args.reps, args.warmup)
            rec[name] = {"local_us": t_local, "push_us": t_push, "local_tflops": flops / t_local / 1e6,
                         "push_remote_gbs": remote_bytes / t_push / 1e3}
        print(json.dumps(rec), flush=True)
        del remote
    if C.device_status() != 0:
        raise SystemExit("device status word set: a kernel wait timed out")


def quant_bench(args, dev):
    """amax (2 B/element read) and quantize (2 B read + 1 B written per element) on the
    tensors one GMLP step quantises; prints algorithmic GB/s per tensor."""
    T, d, h = args.tokens, args.d, args.hidden
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    for name, shape, fmt in (("x", (T, d), C.E4M3), ("Wf", (2, d, h), C.E4M3), ("H", (T, h), C.E4M3),
                             ("dUG", (2, T, h), C.E5M2)):
        x = torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)
        n = x.numel()
        amax = ops.amax(x)
        for _ in range(args.warmup):
            ops.amax(x)
            ops.quantize(x, fmt, amax)
        torch.cuda.synchronize()
        res = {}
        for kind, fn, nbytes in (("amax", lambda: ops.amax(x), 2 * n), ("quantize", lambda: ops.quantize(x, fmt, amax), 3 * n)):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.reps):
                fn()
            e.record()
            torch.cuda.synchronize()
            us = s.elapsed_time(e) * 1000.0 / args.reps
            res[kind] = {"us": us, "gbs": nbytes / us / 1e3}
        print(json.dumps({"tensor": name, "elements": n, **res}), flush=True)
        del x


def norm_bench(args, dev):
    """RMSNorm on [tokens, d]: fused with the e4m3 quantisation (5 B/element), bf16 output
    (4 B/element) and the backward with a vector scale (6 B/element); algorithmic GB/s."""
    T, d = args.tokens, args.d
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    x = (torch.randn((T, d), generator=gen, device=dev) * 2).to(torch.bfloat16)
    dy = (torch.randn((T, d), generator=gen, device=dev) * 1e-2).to(torch.bfloat16)
    scale = (1 + 0.1 * torch.randn(d, generator=gen, device=dev)).to(torch.bfloat16)
    _, rstd = ops.rmsnorm(x, scale, False, 1e-6)
    n = T * d
    res = {}
    for kind, fn, nbytes in (("norm_quant", lambda: ops.rmsnorm_quant(x, scale, False, 1e-6, C.E4M3), 5 * n),
                             ("norm", lambda: ops.rmsnorm(x, scale, False, 1e-6), 4 * n),
                             ("norm_bwd", lambda: ops.rmsnorm_backward(x, scale, False, rstd, dy), 6 * n)):
        us = _time_us(fn, args.reps, args.warmup)
        res[kind] = {"us": us, "gbs": nbytes / us / 1e3}
    print(json.dumps({"tokens": T, "d": d, **res}), flush=True)


def xent_bench(args, dev):
    """Cross-entropy kernels on [tokens, vocab] bf16 logits: the row pass (2 B/element), the
    combine of 128-column partials, and the backward to e5m2 and to bf16 (2 B read + 1 or 2 B
    written per element); algorithmic GB/s."""
    T, V = args.tokens, args.vocab
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    logits = (torch.randn((T, V), generator=gen, device=dev) * 3).to(torch.bfloat16)
    labels = torch.randint(0, V, (T,), generator=gen, device=dev, dtype=torch.int32)
    dloss = torch.randn((T,), generator=gen, device=dev)
    lse, _, qrow = ops.xent_rows(logits, labels, None)
    groups = (V + 127) // 128
    stats = torch.rand((T, groups, 2), generator=gen, device=dev)
    n = T * V
    res = {}
    for kind, fn, nbytes in (
            ("rows", lambda: ops.xent_rows(logits, labels, None), 2 * n),
            ("combine", lambda: ops.xent_combine(stats, logits, V, labels, None), 8 * T * groups),
            ("grad_e5m2", lambda: ops.xent_grad(logits, labels, None, lse, qrow, dloss, 0.0, C.E5M2), 3 * n),
            ("grad_e5m2_cap", lambda: ops.xent_grad(logits, labels, None, lse, qrow, dloss, 15.0, C.E5M2), 3 * n),
            ("grad_bf16", lambda: ops.xent_grad(logits, labels, None, lse, qrow, dloss, 0.0, C.BF16), 4 * n)):
        us = _time_us(fn, args.reps, args.warmup)
        res[kind] = {"us": us, "gbs": nbytes / us / 1e3}
    print(json.dumps({"tokens": T, "vocab": V, **res}), flush=True)


def ns_bench(args, dev):
    """Newton-Schulz (ufp8_newton_schulz) on [batch, d, hidden] f32 slices, 5 'muon' steps;
    algorithmic TF/s = 5 (4 s^2 l + 2 s^3) per slice / time."""
    from .muon import ns_coefficients
    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    g = torch.randn((args.batch, args.d, args.hidden), generator=gen, device=dev)
    co = ns_coefficients(5, "muon")
    s_, l_ = min(args.d, args.hidden), max(args.d, args.hidden)
    fl = args.batch * 5 * (4.0 * s_ * s_ * l_ + 2.0 * s_ ** 3)
    us = _time_us(lambda: ops.newton_schulz(g, co), args.reps, args.warmup)
    print(json.dumps({"batch": args.batch, "m": args.d, "n": args.hidden, "us": us, "tflops": fl / us / 1e6}),
          flush=True)


def attn_bench(args, dev):
    """Causal segment-masked GQA attention (softmax_attention) forward and backward on
    [batch, seq, kv_heads * group, head_dim] bf16, default positions.  Algorithmic TF/s counts the
    causal half of each product, 2 b hi n^2 d / 2 FLOP: two in the forward (Q K^T, P V; the fused
    path runs the score product twice, counted once) and four in the backward (dP, dQ, dK, dV)."""
    from .attention import softmax_attention
    b, n, H, I, dh = args.batch, args.seq, args.kv_heads, args.group, args.head_dim
    gen = torch.Generator(device=dev)
    gen.manual_seed(8)
    mk = lambda shape: torch.randn(shape, generator=gen, device=dev).to(torch.bfloat16)  # noqa: E731
    q = mk((b, n, H * I, dh)).requires_grad_(True)
    k = mk((b, n, H, dh)).requires_grad_(True)
    v = mk((b, n, H, dh)).requires_grad_(True)
    do = mk((b, n, H * I, dh))
    seg = torch.zeros((b, n), dtype=torch.int32, device=dev)
    box = {}

    def fwd():
        box["o"] = softmax_attention(q, k, v, None, seg, None, seg, scale=dh ** -0.5)

    def bwd():
        q.grad = k.grad = v.grad = None
        box["o"].backward(do, retain_graph=True)

    fwd()
    us_f = _time_us(fwd, args.reps, args.warmup)
    us_b = _time_us(bwd, args.reps, args.warmup)
    fl = 2.0 * b * H * I * n * n * dh / 2  # one causal product
    print(json.dumps({"batch": b, "seq": n, "q_heads": H * I, "kv_heads": H, "head_dim": dh, "fwd_us": us_f,
                      "bwd_us": us_b, "fwd_tflops": 2 * fl / us_f / 1e6, "bwd_tflops": 4 * fl / us_b / 1e6}),
          flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=14336)
    ap.add_argument("--gemms", default=",".join(ALL))
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--variant", type=int, default=0, help="0 auto, 1 one CTA per tile, 2 CTA pair, 3 CTA pair with direct stores")
    ap.add_argument("--seconds", type=float, default=0.0, help="sustained loop length per GEMM (0 = off)")
    ap.add_argument("--cublas", action="store_true", help="also time cuBLAS fp8 GEMMs of the same shapes")
    ap.add_argument("--group-m", type=int, default=0, help="tile raster group (0 = library default)")
    ap.add_argument("--quant", action="store_true", help="time amax and quantize on the GMLP tensor sizes instead")
    ap.add_argument("--norm", action="store_true", help="time the RMSNorm kernels on [tokens, d] instead")
    ap.add_argument("--xent", action="store_true", help="time the cross-entropy kernels on [tokens, vocab] instead")
    ap.add_argument("--vocab", type=int, default=128256)
    ap.add_argument("--ns", action="store_true", help="time Newton-Schulz on [batch, d, hidden] instead")
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--attn", action="store_true",
                    help="time the causal attention fwd / bwd on [batch, seq, kv_heads x group, head_dim] instead")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--group", type=int, default=4)
    ap.add_argument("--head-dim", type=int, default=128)
    ap.add_argument("--rs-push", action="store_true",
                    help="time the TP-2/4/8 F2 and B4 GEMMs storing locally vs pushing rows to a peer GPU")
    args = ap.parse_args()
    C.set_gemm_raster(args.group_m)
    C.set_gemm_variant(args.variant)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    if args.quant:
        return quant_bench(args, dev)
    if args.norm:
        return norm_bench(args, dev)
    if args.xent:
        return xent_bench(args, dev)
    if args.ns:
        return ns_bench(args, dev)
    if args.attn:
        return attn_bench(args, dev)
    if args.rs_push:
        return rs_push_bench(args, dev)
    g = build(args.tokens, args.d, args.hidden, dev)
    names = [n.strip() for n in args.gemms.split(",") if n.strip()]
    for n in names:
        if n not in g:
            raise SystemExit(f"unknown GEMM {n}; choose from {ALL}")
    if args.cublas:
        cb = cublas_same_shapes(args.tokens, args.d, args.hidden, dev)
        g.update(cb)
        names += list(cb)
    for n in names:  # warm-up, in order
        for _ in range(args.warmup):
            g[n][1]()
    torch.cuda.synchronize()
    for n in names:
        flops, fn = g[n]
        rec = {"gemm": n, "variant": args.variant, "group_m": args.group_m, "tokens": args.tokens, "d": args.d, "hidden": args.hidden}
        if args.seconds > 0:
            ms, mhz, power, samples = sustained(fn, args.seconds, 0)
            rec.update(us=ms * 1000.0, tflops=flops / ms / 1e9, sm_mhz_median=mhz, power_w_max=power,
                       clock_samples=samples, seconds=args.seconds)
        else:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(args.reps):
                fn()
            e.record()
            torch.cuda.synchronize()
            us = s.elapsed_time(e) * 1000.0 / args.reps
            rec.update(us=us, tflops=flops / us / 1e6)
        print(json.dumps(rec), flush=True)
    if C.device_status() != 0:
        raise SystemExit("device status word set: a kernel wait timed out")


if __name__ == "__main__":
    main()
