#!/usr/bin/env python
"""FP8 GMLP forward + backward benchmark (one JSON line on rank 0).

Workload: the tensor-parallel GMLP block of macrogpt-jax at d_model 4096, hidden 14336,
16384 tokens (B 4 x S 4096) per step, FP8 (e4m3 forward operands, e5m2 gradients, fp32
accumulate, bf16 outputs), seeded synthetic inputs: x ~ N(0, 1), dY ~ N(0, 1e-3),
weights ~ N(0, 1/fan_in).  A step is one forward and one backward pass of the block
through the public module API (GMLP(...)(x).backward(dY)); at N GPUs the same 16384-token
step runs tensor-parallel over N ranks (strong scaling).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the CPU oracle of the same path (the reference's own program is
JAX, which cannot be installed on these machines) on the host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "FP8 GMLP fwd+bwd TFLOP/s/GPU (% of FP8 peak), tokens/s at 1/2/4/8 B200"
CONFIGS = {
    # the tensor-parallel GMLP workload (headline), the small single-GPU GMLP, and the
    # attention projections (fused QKV d -> 3d plus O d -> d, 16 heads x 128)
    "gmlp_d4096": dict(kind="gmlp", d=4096, h=14336, B=4, S=4096),
    "gmlp_d768": dict(kind="gmlp", d=768, h=3072, B=8, S=1024),
    # the MLP half of a transformer layer at the headline sizes: RMSNorm (fused with the fp8
    # quantisation of its output) -> GMLP, forward and backward
    "norm_gmlp_d4096": dict(kind="gmlp", d=4096, h=14336, B=4, S=4096, norm=True),
    "attn_d2048": dict(kind="attn", d=2048, heads=16, head_d=128, B=16, S=1024),
    # the output head of the Llama-3-8B shape (final RMSNorm, lm_head 4096 -> 128256, soft cap) and
    # the next-token loss, forward and backward, on one GPU
    "head_xent_v128256": dict(kind="head", d=4096, V=128256, B=4, S=4096),
    # Muon's Newton-Schulz orthogonalisation of one GMLP block's gradients at d 4096 / h 14336:
    # the fused weight's two [4096, 14336] slices and the down weight [14336, 4096], f32 in and out
    "muon_ns_d4096_h14336": dict(kind="muon", d=4096, h=14336, steps=5),
    # one Llama-3-8B transformer layer (ueaj/model/layer.py:40-58): RMSNorm -> FP8 q/k/v projections
    # (32 query heads in 8 groups of 4, head 128) -> RoPE -> causal softmax attention -> FP8 o
    # projection, then RMSNorm -> FP8 GMLP (h 14336); forward and backward on one GPU
    "layer_llama3_8b": dict(kind="layer", d=4096, h=14336, kv_heads=8, group=4, head_d=128, B=4, S=4096),
}
FP8_NOMINAL_TFLOPS = 4500.0  # B200 dense FP8 datasheet figure
GMLP_D4096_GEMM_TRAFFIC = 1.651e9  # DRAM bytes per GEMM launch, T 16384 / d 4096 / h 14336, from one ncu
# capture of kernel_bench with this build's kernels (profiles/gemm_dram_traffic_d4096_t16384.md)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def flops_per_step(T, d, h):
    """Algorithmic GMLP fwd+bwd FLOPs: 18 T d h (F1 4Tdh, F2 2Tdh, backward twice that)."""
    return 18.0 * T * d * h


def attn_flops_per_step(T, d):
    """Attention projections fwd+bwd: QKV 2 T d 3d + O 2 T d d forward, twice that backward."""
    return 3.0 * (2.0 * T * d * 3 * d + 2.0 * T * d * d)


def head_flops_per_step(T, d, V):
    """lm_head fwd+bwd: logits 2 T d V, dX 2 T d V, dW 2 T d V (the reference's rematerialised
    recomputation of the logits in its backward is not counted)."""
    return 6.0 * T * d * V


def ns_flops(m, n, steps):
    """Newton-Schulz on one [m, n] slice: per step X X^T (2 s^2 l), A A (2 s^3), B X (2 s^2 l)
    with s = min(m, n), l = max(m, n)."""
    s_, l_ = min(m, n), max(m, n)
    return steps * (4.0 * s_ * s_ * l_ + 2.0 * s_ ** 3)


def layer_flops(cfg, T, S, B):
    """Algorithmic FLOPs of one layer fwd+bwd: GMLP 18 T d h; projections 3 x 2 T d (q + k + v + o
    widths); causal attention 3 x 2 x 2 B HI S^2 Dh / 2 (QK^T and PV forward, four products backward,
    half the score matrix visible)."""
    d, h, H, I, Dh = cfg["d"], cfg["h"], cfg["kv_heads"], cfg["group"], cfg["head_d"]
    proj = 3.0 * 2.0 * T * d * (2 * H * I * Dh + 2 * H * Dh)
    attn = 3.0 * 2.0 * 2.0 * B * H * I * S * S * Dh / 2.0
    return 18.0 * T * d * h + proj + attn, proj, attn


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured (MEASURED_PEAKS.json)"
        except Exception:
            pass
    return dict(FALLBACK_PEAKS), "fallback (earlier measurement on this pool)"


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampled every 50 ms while the timed region runs; start() returns once the
    first sample has been written (at most 2 s), so the samples cover the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 2.0 and self.proc.poll() is None:
            if os.path.getsize(self.path) > 0:
                break
            time.sleep(0.01)

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.06)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = [r.split(", ") for r in Path(self.path).read_text().strip().splitlines() if r.strip()]
        os.unlink(self.path)
        rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].strip().lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit()),
                "reasons": reasons, "samples": len(rows)}


# ----------------------------------------------------------------------------- CPU baseline
def cpu_oracle_step(d, h, T, seed=0):
    """Seconds the oracle takes for one GMLP fwd+bwd step of T tokens on the host: per-tensor
    quantisation (and dequantisation) of the weights, both contractions forward, the four
    backward, gating and the activation/gradient quantisations."""
    import numpy as np
    from oracle import fp8 as ofp8
    from oracle import path as op
    op.FAST_CAST = True
    ofp8.THREADED = True
    rng = np.random.default_rng(seed)
    wf = op.bf16_normal(rng, (2, d, h), d ** -0.5)
    wd = op.bf16_normal(rng, (h, d), h ** -0.5)
    x = op.bf16_normal(rng, (T, d))
    dy = op.bf16_normal(rng, (T, d), 1e-3)
    t0 = time.perf_counter()
    _, saved = op.gmlp_forward(x, wf, wd, acc=np.float32)
    op.gmlp_backward(dy, saved, acc=np.float32)
    return time.perf_counter() - t0


def cpu_head_step(d, V, T, seed=0):
    """Seconds the oracle takes for one output-head step of T tokens over V classes on the host,
    as (activation side, weight quantisation): the first is norm + fp8 quantisation, logits, soft
    cap, loss, fp8 logit gradient, the two backward contractions and the norm backward; the second
    the e4m3 quantisation of the [d, V] weight (independent of T)."""
    import numpy as np
    from oracle import fp8 as ofp8
    from oracle import path as op
    from oracle import xent as ox
    op.FAST_CAST = True
    ofp8.THREADED = True
    rng = np.random.default_rng(seed)
    w = op.bf16_normal(rng, (d, V), d ** -0.5)
    x = op.bf16_normal(rng, (T, d))
    scale = op.bf16_normal(rng, (d,), 0.1)
    labels = rng.integers(0, V, T).astype(np.int32)
    t0 = time.perf_counter()
    qw = op.quant(w, ofp8.E4M3)
    t1 = time.perf_counter()
    _, saved = ox.head_forward(x, scale, False, 1e-6, qw, labels, None, 15.0, acc=np.float32)
    ox.head_backward(np.ones(T, np.float32), saved, x, scale, False, labels, None, 15.0, acc=np.float32)
    return time.perf_counter() - t1, t1 - t0


CPU_VOCAB_SLICES = (1024, 4096)  # vocabulary widths the CPU port executes for the head workload
CPU_HEAD_TOKENS = 4096  # tokens per executed CPU head step


def head_cpu_estimate(d, V, T, samples):
    """Full-config seconds from executed head steps [(V slice, t_act, t_wq)] at CPU_HEAD_TOKENS
    tokens: t = (T / Ts) (a + b V) + c V, with a + b V fitted to the activation-side times (all of
    that work is per token) and c the weight quantisation time per vocabulary column."""
    act, a, b = fit_hidden([(vs, ta) for vs, ta, _ in samples], V)
    c = sum(tw / vs for vs, _, tw in samples) / len(samples)
    return (T / CPU_HEAD_TOKENS) * act + c * V, a, b, c


def fit_hidden(samples, h_full):
    """Least-squares fit t(h) = a + b h over (hidden slice, seconds) samples taken at the full
    token count and d_model, evaluated at h_full.  The activation-side work (x and dY
    quantisation, dx rounding) is the intercept a; every weight-side cost is linear in the
    hidden width.  Returns (seconds at h_full, a, b)."""
    import numpy as np
    hs = np.array([s[0] for s in samples], dtype=np.float64)
    ts = np.array([s[1] for s in samples], dtype=np.float64)
    if len(set(hs.tolist())) > 1:
        b, a = np.polyfit(hs, ts, 1)
    else:
        a, b = 0.0, ts.mean() / hs.mean()
    a, b = max(float(a), 0.0), max(float(b), 0.0)
    return a + b * h_full, a, b


CPU_SLICES = (128, 768)  # hidden widths the CPU port executes (alternating), full tokens and d_model


def cpu_sample_desc(T, d, h, n_steps):
    return (f"{n_steps} oracle GMLP fwd+bwd steps at the full {T} tokens and d_model {d} on hidden slices "
            f"{CPU_SLICES[0]} and {CPU_SLICES[1]} (alternating) of {h}, weights quantised each step; fitted as "
            f"t(h) = a + b*h and evaluated at hidden {h}; numpy fp32 BLAS contractions on all host threads, "
            "ml_dtypes casts, single-threaded elementwise")


def head_sample_desc(T, d, V, n_steps):
    return (f"{n_steps} oracle output-head fwd+bwd steps at {CPU_HEAD_TOKENS} of the {T} tokens, d_model {d}, on "
            f"vocabulary slices {CPU_VOCAB_SLICES[0]} and {CPU_VOCAB_SLICES[1]} (alternating) of {V}, weight "
            f"quantised each step (timed apart); estimated as (T / {CPU_HEAD_TOKENS}) (a + b V) + c V at "
            f"T {T}, V {V}; numpy fp32 BLAS contractions on all host threads, ml_dtypes casts")


def cpu_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def gpu_arm_config(args, cfg, world):
    """The `config` dict both arms print for this workload and GPU count."""
    d, h, T = cfg["d"], cfg["h"], cfg["B"] * cfg["S"]
    if world > 1:
        rs = {"auto": "y pushed from the GEMM epilogue, dx by copy engines beside dWf",
              "epilogue": "pushed from the GEMM epilogues", "copy": "by copy engines"}[args.tp_rs_engine]
        parallelism = (f"tp{world} (NVLink P2P; all-gather consumed block by block by the GEMMs, by "
                       f"{'SM push kernel' if args.tp_ag == 'sm' else 'copy engines'}"
                       f"{'' if args.tp_lanes == 1 or args.tp_ag == 'sm' else f' on {args.tp_lanes} lanes'}; "
                       f"reduce-scatter {rs})" if args.tp_rs == "p2p"
                       else f"tp{world} (NCCL all-gather / reduce-scatter / all-reduce)")
    else:
        parallelism = "tp1"
    return {"workload": args.config_desc, "tokens": T, "d_model": d, "hidden": h, "parallelism": parallelism,
            "l2": ("inputs larger than L2" if T * (6 * h + 3 * d) * 2 > 2 * 126e6 else
                   "working set below 2x L2: no flush between steps (secondary workload)")}


# ----------------------------------------------------------------------------- arms
def head_arm_config(args, cfg):
    d, V, T = cfg["d"], cfg["V"], cfg["B"] * cfg["S"]
    return {"workload": args.config_desc, "tokens": T, "d_model": d, "vocab": V, "parallelism": "tp1",
            "l2": "inputs larger than L2"}


def run_reference(args, cfg, rank, world):
    """The CPU port of the path (oracle/), rank 0 only.  Every step runs the full token count
    on a hidden slice (the head workload: a vocabulary slice); the printed ms_per_step is the
    measured time of those executed steps, and `value` is the full-config throughput from the
    fit t(h) = a + b h (fields `executed` and `extrapolation` give both)."""
    if rank != 0:
        return None
    head = cfg["kind"] == "head"
    d, T = cfg["d"], cfg["B"] * cfg["S"]
    h = cfg["V"] if head else cfg["h"]
    slices = CPU_VOCAB_SLICES if head else CPU_SLICES
    samples, head_samples = [], []
    for i in range(args.warmup + args.steps):
        hs = slices[i % 2]
        if head:
            ta, tw = cpu_head_step(d, hs, CPU_HEAD_TOKENS, seed=i)
            t = ta + tw
        else:
            t = cpu_oracle_step(d, hs, T, seed=i)
        if i >= args.warmup:
            samples.append((hs, t))
            if head:
                head_samples.append((hs, ta, tw))
    if head:
        full_s, a, b, c = head_cpu_estimate(d, h, T, head_samples)
    else:
        full_s, a, b = fit_hidden(samples, h)
    exec_ms = 1000.0 * sum(s[1] for s in samples) / len(samples)
    value = T / full_s
    by_h = {str(hs): 1000.0 * sum(s[1] for s in samples if s[0] == hs) / max(1, sum(1 for s in samples if s[0] == hs))
            for hs in slices}
    out = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": exec_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp8",
        "data": "synthetic (seeded)",
        "config": head_arm_config(args, cfg) if head else gpu_arm_config(args, cfg, world),
        "tflops_per_gpu": (head_flops_per_step(T, d, h) if head else flops_per_step(T, d, h)) / full_s / 1e12,
        "executed": {"steps": args.steps, "warmup_steps": args.warmup, "tokens": T, "d_model": d,
                     ("vocab_slices" if head else "hidden_slices"): list(slices), "ms_per_step": exec_ms,
                     "ms_per_step_by_slice": by_h,
                     "note": "ms_per_step is the mean measured time of these executed steps"},
        "extrapolation": {"model": ("t = (T / Ts) (a + b V) + c V; a, b least squares over the executed steps' "
                                    "activation-side times, c their weight quantisation time per column") if head
                          else "t(h) = a + b*h, least squares over the executed steps",
                          "a_ms": 1000.0 * a, "b_ms_per_hidden": 1000.0 * b, "to_hidden": h,
                          "est_ms_per_step_full": 1000.0 * full_s, "factor": 1000.0 * full_s / exec_ms,
                          "note": "value (tokens/s) = tokens / est_ms_per_step_full: an estimate for the full "
                                  "config, not a measurement of it"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                         "sample": head_sample_desc(T, d, h, args.steps) if head else
                         cpu_sample_desc(T, d, h, args.steps)},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    return out


def e2e_pipelined(step_fn, x_in, dy_in, steps, barrier, graph=False, y_like=None):
    """Milliseconds for `steps` end-to-end steps: each step's x and dY are copied from pinned
    host memory into one of two device buffers on a copy stream (the copy for step i+1 runs
    while step i computes), and each step's y is copied back to pinned host memory on a second
    copy stream as soon as the forward has produced it.  step_fn(x, dy) -> (y, event after
    which y is final, or None for the end of the step).  Timed with CUDA events on the compute
    stream, which waits for both copy streams before the end event.  y_like: a tensor of y's shape
    and dtype (default: x's shape in bf16)."""
    import torch
    cur = torch.cuda.current_stream()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    x_host = x_in.cpu().pin_memory()
    dy_host = dy_in.cpu().pin_memory()
    xb = [torch.empty_like(x_in) for _ in range(2)]
    dyb = [torch.empty_like(dy_in) for _ in range(2)]
    if y_like is None:
        yh = [torch.empty(x_in.shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    else:
        yh = [torch.empty(y_like.shape, dtype=y_like.dtype).pin_memory() for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    buf_free = [torch.cuda.Event() for _ in range(2)]
    y_done = [torch.cuda.Event() for _ in range(2)]

    def issue_h2d(i):
        b = i % 2
        with torch.cuda.stream(h2d):
            if i >= 2:
                h2d.wait_event(buf_free[b])
            xb[b].copy_(x_host, non_blocking=True)
            dyb[b].copy_(dy_host, non_blocking=True)
            in_ready[b].record(h2d)

    def run_steps(n):
        issue_h2d(0)
        for i in range(n):
            b = i % 2
            if i + 1 < n:
                issue_h2d(i + 1)
            cur.wait_event(in_ready[b])
            if graph and i >= 1:
                cur.wait_event(y_done[(i - 1) % 2])  # a replay overwrites the previous step's y
            y, y_ev = step_fn(xb[b], dyb[b])
            buf_free[b].record(cur)
            with torch.cuda.stream(d2h):
                d2h.wait_event(y_ev if y_ev is not None else buf_free[b])
                yh[b].copy_(y.detach(), non_blocking=True)
                y_done[b].record(d2h)
            if not graph:
                y.record_stream(d2h)  # the allocator must not hand y out again before the copy
        cur.wait_stream(h2d)
        cur.wait_stream(d2h)

    run_steps(2)  # warm-up of the copy path
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(cur)
    h2d.wait_stream(cur)
    d2h.wait_stream(cur)
    run_steps(steps)
    e1.record(cur)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1)


def tp_parity_check(mlp, x_full, dy_full, x_in, dy_in, d, h, rank, world, dev):
    """One tensor-parallel step (outside any timed region) against the single-GPU GMLP with the
    same weights and inputs on rank 0: y and dx gathered over tokens, dWf and dWd gathered over
    the hidden axis.  Returns {tensor: {max_rel, cos}} on rank 0 (None elsewhere).  The two
    differ only in the order of the final bf16 sums (every per-tensor scale is global)."""
    import torch
    import torch.distributed as dist
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP
    xl = x_in.detach().requires_grad_(True)
    y = mlp(xl)
    y.backward(dy_in)
    torch.cuda.synchronize()
    dist.barrier()

    def gather(t, dim):
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return torch.cat(parts, dim=dim)

    got = {"y": gather(y.detach(), 0), "dx": gather(xl.grad, 0),
           "dWf": gather(mlp.fused_proj.w.grad, 2), "dWd": gather(mlp.down_proj.w.grad, 0)}
    for p in mlp.parameters():
        p.grad = None
    if rank != 0:
        return None
    ref_mlp = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(d ** -0.5)),
                            down_proj=Einsum.override(initializer=scaled_normal_init(h ** -0.5)))(
        model_d=d, hidden_d=h, rngs=Rngs(0))
    xr = x_full.reshape(-1, d).detach().requires_grad_(True)
    yr = ref_mlp(xr)
    yr.backward(dy_full.reshape(-1, d))
    ref = {"y": yr.detach(), "dx": xr.grad, "dWf": ref_mlp.fused_proj.w.grad, "dWd": ref_mlp.down_proj.w.grad}
    out = {"vs": "single-GPU GMLP on rank 0, same weights and inputs"}
    for k in ("y", "dx", "dWf", "dWd"):
        a, b = got[k].double().reshape(-1), ref[k].double().reshape(-1)
        out[k] = {"max_rel": float((a - b).abs().max() / b.abs().max()),
                  "cos": float(torch.dot(a, b) / (a.norm() * b.norm()))}
    del ref_mlp
    return out


def run_ours(args, cfg, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from macrogpt_jax_b200 import _capi, ops
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    _capi.set_gemm_variant(args.gemm_variant)
    if cfg["kind"] == "attn":
        return run_attn(args, cfg, rank, world, local_rank, dev)
    if cfg["kind"] == "head":
        return run_head(args, cfg, rank, world, local_rank, dev)
    if cfg["kind"] == "muon":
        return run_muon(args, cfg, rank, world, local_rank, dev)
    if cfg["kind"] == "layer":
        return run_layer(args, cfg, rank, world, local_rank, dev)
    d, h, B, S = cfg["d"], cfg["h"], cfg["B"], cfg["S"]
    T = B * S
    if world > 1 and cfg.get("norm"):
        raise SystemExit("the RMSNorm -> GMLP workload runs on one GPU")
    if world > 1:
        from macrogpt_jax_b200 import tp as tp_mod
        from macrogpt_jax_b200.tp import TPGMLP
        tp_mod.AG_ENGINE = _capi.AG_SM if args.tp_ag == "sm" else _capi.AG_COPY_ENGINE
        tp_mod.COPY_LANES = args.tp_lanes
        tp_mod.RS_ENGINE = args.tp_rs_engine
        mlp = TPGMLP(model_d=d, hidden_d=h, rngs=Rngs(0), device=dev,
                     fused_init=scaled_normal_init(d ** -0.5), down_init=scaled_normal_init(h ** -0.5),
                     fused_reduce_scatter=args.tp_rs == "p2p")
    else:
        mlp = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(d ** -0.5)),
                            down_proj=Einsum.override(initializer=scaled_normal_init(h ** -0.5)))(
            model_d=d, hidden_d=h, rngs=Rngs(0))
        assert mlp.fused()
    block = mlp
    if cfg.get("norm"):
        from macrogpt_jax_b200.layer import norm_fusable, norm_mlp
        from macrogpt_jax_b200.rmsnorm import RMSNorm
        norm = RMSNorm(d, rngs=Rngs(1), device=dev)
        assert norm_fusable(norm, mlp)
        if args.norm_unfused:
            block = lambda t: mlp(norm(t))  # noqa: E731
        else:
            block = lambda t: norm_mlp(norm, mlp, t)  # noqa: E731
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)  # identical activations on every rank (TP replicates x and dY)
    x_full = torch.randn((B, S, d), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    dy_full = (torch.randn((B, S, d), generator=gen, device=dev, dtype=torch.float32) * 1e-3).to(torch.bfloat16)
    x_in, dy_in = (mlp.shard_tokens(x_full), mlp.shard_tokens(dy_full)) if world > 1 else (x_full, dy_full)
    params = list(mlp.parameters()) + (list(norm.parameters()) if cfg.get("norm") else [])

    def step(xb, dyb):
        xl = xb.detach().requires_grad_(True)
        y = block(xl)
        y.backward(dyb)
        for p in params:
            p.grad = None
        return y

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        step(x_in, dy_in)
    torch.cuda.synchronize()
    barrier()
    run = step
    if args.graph:
        if world > 1:
            raise SystemExit("--graph runs on one GPU (the tensor-parallel path is not capturable)")
        from macrogpt_jax_b200.graphs import GraphedStep
        run = GraphedStep(step, x_in, dy_in, warmup=args.warmup)
        torch.cuda.synchronize()

    # ---- headline: device-resident inputs, per-launch events on the launching stream
    timer = ops.KernelTimer()
    clocks = ClockSampler(local_rank)
    clocks.start()
    launches0 = _capi.launches
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if not args.graph:
        ops.set_timer(timer)
    ev0.record()
    for _ in range(args.steps):
        run(x_in, dy_in)
    ev1.record()
    ops.set_timer(None)
    torch.cuda.synchronize()
    barrier()
    launches = _capi.launches - launches0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    eager_ms = ms
    if args.graph:
        # Per-kernel CUDA events cannot be recorded inside a graph: the kernel shares and the
        # roofline come from an eager pass of the same step right after the graph-timed region.
        launches0 = _capi.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ops.set_timer(timer)
        e0.record()
        for _ in range(args.steps):
            step(x_in, dy_in)
        e1.record()
        ops.set_timer(None)
        torch.cuda.synchronize()
        launches = _capi.launches - launches0  # the graph replays exactly these kernels
        eager_ms = e0.elapsed_time(e1)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    summ = timer.summary()

    # ---- end to end: host (pinned) inputs copied in and y read back inside the timed region
    e2e = None
    if not args.no_e2e:
        if args.graph:
            def split_step(xb, dyb):
                return run(xb, dyb), None
        else:
            def split_step(xb, dyb):
                # y can leave for the host as soon as the forward has produced it, while the
                # backward of the same step runs.
                xl = xb.detach().requires_grad_(True)
                y = block(xl)
                y_ev = torch.cuda.Event()
                y_ev.record()
                y.backward(dyb)
                for p in params:
                    p.grad = None
                return y, y_ev
        ems = e2e_pipelined(split_step, x_in, dy_in, args.steps, barrier, graph=args.graph)
        ems_t = torch.tensor([ems], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems_t, op=dist.ReduceOp.MAX)
        ems = float(ems_t.item())
        nb = x_in.numel() * 2
        e2e = {"value": T * args.steps / (ems / 1000.0), "unit": "tokens/s", "ms_per_step": ems / args.steps,
               "h2d_bytes_per_step": 2 * nb * world, "d2h_bytes_per_step": nb * world,
               "path": "GMLP module forward+backward; every step copies its x and dY from pinned host memory "
                       "(side stream, double-buffered: step i+1's inputs arrive while step i computes) and "
                       "reads its y back (side stream, overlapping the backward)"}

    tp_parity = None
    if world > 1 and not args.no_tp_parity:
        tp_parity = tp_parity_check(mlp, x_full, dy_full, x_in, dy_in, d, h, rank, world, dev)

    if rank != 0:
        return None
    peaks, peak_src = load_peaks()
    fl = flops_per_step(T, d, h)
    traffic, traffic_src = args.gemm_traffic, "--gemm-traffic" if args.gemm_traffic else None
    if traffic is None and args.config == "gmlp_d4096" and world == 1:
        # Mean dram__bytes_read.sum + dram__bytes_write.sum per GEMM launch over the six
        # contractions of this workload, from one ncu capture of kernel_bench at these sizes.
        traffic, traffic_src = GMLP_D4096_GEMM_TRAFFIC, ("past ncu capture (not measured by this run): mean "
                                                         "dram__bytes_read + write of the six GEMMs of this workload, "
                                                         "kernel_bench at these sizes")
    tokens_s = T * args.steps / (ms / 1000.0)
    tflops_gpu = fl * args.steps / (ms / 1000.0) / world / 1e12
    g_n, g_ms, g_fl = summ.get("gemm", (0, 0.0, 0.0))
    peak_fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    achieved = (g_fl / g_n) / (g_ms / g_n / 1000.0) / 1e12 if g_n else None
    q_n, q_ms, q_b = summ.get("quantize", (0, 0.0, 0.0))
    a_n, a_ms, a_b = summ.get("amax", (0, 0.0, 0.0))
    out = {
        "metric": METRIC, "value": tokens_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp8", "data": "synthetic (seeded)",
        "config": gpu_arm_config(args, cfg, world),
        "tflops_per_gpu": tflops_gpu,
        "frac_of_fp8_peak": {"nominal_4500": tflops_gpu / FP8_NOMINAL_TFLOPS,
                             "measured_2x_bf16_sustained": tflops_gpu / peak_fp8},
        "roofline": {"kernel": "gemm_fp8_pair_kernel", "bound": "tensor", "achieved": achieved,
                     "peak": peak_fp8, "unit": "TFLOP/s", "frac": (achieved / peak_fp8) if achieved else None,
                     "frac_of_nominal_fp8": (achieved / FP8_NOMINAL_TFLOPS) if achieved else None,
                     "peak_source": f"2 x bf16_tflops_sustained, {peak_src}; tcgen05 runs fp8 at twice "
                                    "its bf16 rate",
                     "launches": g_n, "time_share": g_ms / eager_ms if eager_ms else None,
                     "traffic": traffic, "traffic_source": traffic_src},
        "roofline_quantize": {"bound": "hbm", "unit": "GB/s",
                              "achieved": (q_b / (q_ms / 1000.0) / 1e9) if q_n else None,
                              "peak": peaks["hbm_gbs"],
                              "frac": (q_b / (q_ms / 1000.0) / 1e9 / peaks["hbm_gbs"]) if q_n else None,
                              "launches": q_n, "time_share": q_ms / eager_ms if eager_ms else None,
                              "amax_achieved_gbs": (a_b / (a_ms / 1000.0) / 1e9) if a_n else None,
                              "amax_time_share": a_ms / eager_ms if eager_ms else None},
        "gpu_launches": launches,
        "clocks": clk,
    }
    norm_parts = {k: summ[k] for k in ("norm_quant", "norm", "norm_bwd") if k in summ}
    if norm_parts:
        # algorithmic bytes: norm_quant 5 B/element (x twice, fp8 out), norm 4 B (x, bf16 y),
        # norm_bwd 6 B (x, dy, dx)
        out["roofline_norm"] = {k: {"bound": "hbm", "unit": "GB/s", "launches": n,
                                    "achieved": b / (ms / 1000.0) / 1e9, "peak": peaks["hbm_gbs"],
                                    "frac": b / (ms / 1000.0) / 1e9 / peaks["hbm_gbs"],
                                    "time_share": ms / eager_ms if eager_ms else None}
                                for k, (n, ms, b) in norm_parts.items()}
    if args.graph:
        out["config"]["execution"] = "CUDA graph of the whole step (macrogpt_jax_b200.graphs.GraphedStep)"
        out["roofline"]["source"] = ("per-kernel CUDA events of an eager pass of the same step right after the "
                                     "graph-timed region (events cannot be recorded inside a graph); time_share "
                                     f"is of that pass ({eager_ms / args.steps:.3f} ms/step eager)")
    if e2e:
        out["e2e"] = e2e
    if tp_parity:
        out["tp_parity"] = tp_parity
    if world == 1 and not args.no_cpu_baseline:
        samples = [(hs, cpu_oracle_step(d, hs, T, seed=k)) for k, hs in enumerate(CPU_SLICES)]
        step_s, a, b = fit_hidden(samples, h)
        out["cpu_baseline"] = {"value": T / step_s, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                               "sample": cpu_sample_desc(T, d, h, len(samples)), "est_ms_per_step": step_s * 1000.0,
                               "executed_ms": {str(hs): 1000.0 * s for hs, s in samples},
                               "tflops": flops_per_step(T, d, h) / step_s / 1e12}
    return out


def run_attn(args, cfg, rank, world, local_rank, dev):
    """Attention projections: qkv = fused QKV Einsum(x), y = O Einsum(a), then the backward
    of both with seeded upstream gradients.  The attention kernel between them is not part of
    this library, so `a` is an independent seeded input of the attention-output shape."""
    import torch
    from macrogpt_jax_b200 import _capi, ops
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.soft_attn import SoftmaxAttention
    if world > 1:
        raise SystemExit("the attention-projection workload runs on one GPU")
    d, H, K, B, S = cfg["d"], cfg["heads"], cfg["head_d"], cfg["B"], cfg["S"]
    T = B * S
    init = Einsum.override(initializer=scaled_normal_init(d ** -0.5))
    m = SoftmaxAttention(d, kq_d=K, kv_heads=H, rngs=Rngs(0), fused_qkv=True, qkv=init, o=init)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    rnd = lambda *shape, std=1.0: (torch.randn(shape, generator=gen, device=dev) * std).to(torch.bfloat16)  # noqa
    x, a = rnd(B, S, d), rnd(B, S, H, 1, K)
    dqkv, dy = rnd(3, B, S, H, K, std=1e-3), rnd(B, S, d, std=1e-3)
    params = list(m.parameters())

    def step(xb, ab):
        xl = xb.detach().requires_grad_(True)
        al = ab.detach().requires_grad_(True)
        qkv = m.qkv(xl)
        y = m.project_out(al)
        torch.autograd.backward([qkv, y], [dqkv, dy])
        for p in params:
            p.grad = None
        return y

    for _ in range(args.warmup):
        step(x, a)
    torch.cuda.synchronize()
    run = step
    if args.graph:
        from macrogpt_jax_b200.graphs import GraphedStep
        run = GraphedStep(step, x, a, warmup=args.warmup)
        torch.cuda.synchronize()
    timer = ops.KernelTimer()
    clocks = ClockSampler(local_rank)
    clocks.start()
    launches0 = _capi.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if not args.graph:
        ops.set_timer(timer)
    ev0.record()
    for _ in range(args.steps):
        run(x, a)
    ev1.record()
    ops.set_timer(None)
    torch.cuda.synchronize()
    launches = _capi.launches - launches0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    eager_ms = ms
    if args.graph:  # per-kernel events come from an eager pass (none can be recorded in a graph)
        launches0 = _capi.launches
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ops.set_timer(timer)
        e0.record()
        for _ in range(args.steps):
            step(x, a)
        e1.record()
        ops.set_timer(None)
        torch.cuda.synchronize()
        launches = _capi.launches - launches0
        eager_ms = e0.elapsed_time(e1)
    summ = timer.summary()
    peaks, peak_src = load_peaks()
    fl = attn_flops_per_step(T, d)
    tflops = fl * args.steps / (ms / 1000.0) / 1e12
    g_n, g_ms, g_fl = summ.get("gemm", (0, 0.0, 0.0))
    peak_fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    achieved = (g_fl / g_n) / (g_ms / g_n / 1000.0) / 1e12 if g_n else None
    out = {
        "metric": "FP8 attention projections fwd+bwd tokens/s (TFLOP/s/GPU)", "value": T * args.steps / (ms / 1000.0),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp8", "data": "synthetic (seeded)",
        "config": {"workload": args.config_desc, "tokens": T, "d_model": d, "heads": H, "head_dim": K,
                   "parallelism": "single GPU", "l2": "inputs larger than L2"},
        "tflops_per_gpu": tflops,
        "roofline": {"kernel": "gemm_fp8_pair_kernel", "bound": "tensor", "achieved": achieved, "peak": peak_fp8,
                     "unit": "TFLOP/s", "frac": (achieved / peak_fp8) if achieved else None,
                     "peak_source": f"2 x bf16_tflops_sustained, {peak_src}", "launches": g_n,
                     "time_share": g_ms / eager_ms if eager_ms else None, "traffic": None},
        "gpu_launches": launches, "clocks": clk,
    }
    if args.graph:
        out["config"]["execution"] = "CUDA graph of the whole step (macrogpt_jax_b200.graphs.GraphedStep)"
        out["roofline"]["source"] = ("per-kernel CUDA events of an eager pass of the same step right after the "
                                     "graph-timed region; time_share is of that pass "
                                     f"({eager_ms / args.steps:.3f} ms/step eager)")
    return out


def run_head(args, cfg, rank, world, local_rank, dev):
    """Output head + next-token loss: chunked_softmax_cross_entropy(tokens, x, head.get_logits) with
    an OutputHead (final RMSNorm, FP8 lm_head, soft cap), then the backward of the summed loss."""
    import torch
    from macrogpt_jax_b200 import _capi, ops
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.head import OutputHead
    from macrogpt_jax_b200.next_token_loss import _fused_head, chunked_softmax_cross_entropy
    if world > 1:
        raise SystemExit("the output-head workload runs on one GPU")
    d, V, B, S = cfg["d"], cfg["V"], cfg["B"], cfg["S"]
    T = B * S
    head = OutputHead.override(lm_head=Einsum.override(initializer=scaled_normal_init(d ** -0.5)))(
        d, V, head_cap="tanh", rngs=Rngs(0))
    assert _fused_head(head.get_logits) is head
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    x = torch.randn((B, S, d), generator=gen, device=dev, dtype=torch.float32).to(torch.bfloat16)
    tokens = torch.randint(0, V, (B, S), generator=gen, device=dev, dtype=torch.int64)
    params = list(head.parameters())

    def fwd_bwd(xb, tb):
        xl = xb.detach().requires_grad_(True)
        loss = chunked_softmax_cross_entropy(tb, xl, head.get_logits)
        ev = torch.cuda.Event()
        ev.record()
        loss.sum().backward()
        for p in params:
            p.grad = None
        return loss, ev

    for _ in range(args.warmup):
        fwd_bwd(x, tokens)
    torch.cuda.synchronize()
    timer = ops.KernelTimer()
    clocks = ClockSampler(local_rank)
    clocks.start()
    launches0 = _capi.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ops.set_timer(timer)
    ev0.record()
    for _ in range(args.steps):
        fwd_bwd(x, tokens)
    ev1.record()
    ops.set_timer(None)
    torch.cuda.synchronize()
    launches = _capi.launches - launches0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    summ = timer.summary()

    e2e = None
    if not args.no_e2e:
        ems = e2e_pipelined(fwd_bwd, x, tokens, args.steps, lambda: None, y_like=torch.empty((B, S)))
        e2e = {"value": T * args.steps / (ems / 1000.0), "unit": "tokens/s", "ms_per_step": ems / args.steps,
               "h2d_bytes_per_step": x.numel() * 2 + tokens.numel() * 8, "d2h_bytes_per_step": T * 4,
               "path": "chunked_softmax_cross_entropy(tokens, x, head.get_logits) and the backward of the summed "
                       "loss; every step copies its activations and tokens from pinned host memory (side stream, "
                       "double-buffered) and reads its per-token loss back (side stream, overlapping the backward)"}

    peaks, peak_src = load_peaks()
    fl = head_flops_per_step(T, d, V)
    g_n, g_ms, g_fl = summ.get("gemm", (0, 0.0, 0.0))
    peak_fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    achieved = (g_fl / g_n) / (g_ms / g_n / 1000.0) / 1e12 if g_n else None
    tflops = fl * args.steps / (ms / 1000.0) / 1e12
    hbm = {}
    for k in ("xent_grad", "xent_combine", "quantize", "amax", "norm_quant", "norm_bwd"):
        if k in summ:
            n, kms, b = summ[k]
            hbm[k] = {"bound": "hbm", "unit": "GB/s", "launches": n, "achieved": b / (kms / 1000.0) / 1e9,
                      "peak": peaks["hbm_gbs"], "frac": b / (kms / 1000.0) / 1e9 / peaks["hbm_gbs"],
                      "time_share": kms / ms}
    out = {
        "metric": "FP8 output head + next-token loss fwd+bwd tokens/s (TFLOP/s/GPU)",
        "value": T * args.steps / (ms / 1000.0), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8", "data": "synthetic (seeded)", "config": head_arm_config(args, cfg),
        "tflops_per_gpu": tflops,
        "roofline": {"kernel": "gemm_fp8_pair_kernel", "bound": "tensor", "achieved": achieved, "peak": peak_fp8,
                     "unit": "TFLOP/s", "frac": (achieved / peak_fp8) if achieved else None,
                     "peak_source": f"2 x bf16_tflops_sustained, {peak_src}", "launches": g_n,
                     "time_share": g_ms / ms if ms else None, "traffic": None},
        "roofline_hbm_kernels": hbm,
        "gpu_launches": launches, "clocks": clk,
    }
    if e2e:
        out["e2e"] = e2e
    if not args.no_cpu_baseline:
        samples = [(vs,) + cpu_head_step(d, vs, CPU_HEAD_TOKENS, seed=k) for k, vs in enumerate(CPU_VOCAB_SLICES)]
        step_s, a, b, c = head_cpu_estimate(d, V, T, samples)
        out["cpu_baseline"] = {"value": T / step_s, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                               "sample": head_sample_desc(T, d, V, len(samples)), "est_ms_per_step": step_s * 1000.0,
                               "executed_ms": {str(vs): 1000.0 * (ta + tw) for vs, ta, tw in samples},
                               "tflops": fl / step_s / 1e12}
    return out


def run_muon(args, cfg, rank, world, local_rank, dev):
    """orthogonalize(grad_fused) and orthogonalize(grad_down) (ueaj/opt/multiscale.py:110-141) per
    step, the canonical GMLP weight layouts [2, d, h] and [h, d], f32 in and out."""
    import numpy as np
    import torch
    from macrogpt_jax_b200 import _capi, ops
    from macrogpt_jax_b200.muon import orthogonalize
    if world > 1:
        raise SystemExit("the Newton-Schulz workload runs on one GPU")
    d, h, steps = cfg["d"], cfg["h"], cfg["steps"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    gf = torch.randn((2, d, h), generator=gen, device=dev) * 1e-3
    gd = torch.randn((h, d), generator=gen, device=dev) * 1e-3
    fl = 3 * ns_flops(d, h, steps)

    def step(a, b):
        return orthogonalize(a, ns_steps=steps), orthogonalize(b, ns_steps=steps)

    for _ in range(args.warmup):
        step(gf, gd)
    torch.cuda.synchronize()
    timer = ops.KernelTimer()
    clocks = ClockSampler(local_rank)
    clocks.start()
    launches0 = _capi.launches
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ops.set_timer(timer)
    ev0.record()
    for _ in range(args.steps):
        step(gf, gd)
    ev1.record()
    ops.set_timer(None)
    torch.cuda.synchronize()
    launches = _capi.launches - launches0
    clk = clocks.stop()
    ms = ev0.elapsed_time(ev1)
    summ = timer.summary()
    peaks, peak_src = load_peaks()
    n_n, n_ms, n_fl = summ.get("newton_schulz", (0, 0.0, 0.0))
    achieved = n_fl / (n_ms / 1000.0) / 1e12 if n_n else None
    out = {
        "metric": "Muon Newton-Schulz orthogonalisation TFLOP/s (bf16 tcgen05 GEMMs)",
        "value": fl * args.steps / (ms / 1000.0) / 1e12, "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded)",
        "config": {"workload": args.config_desc, "slices": [[d, h], [d, h], [h, d]], "ns_steps": steps,
                   "parallelism": "single GPU", "l2": "inputs larger than L2"},
        "roofline": {"kernel": "ufp8_newton_schulz (bf16 gemm_fp8_pair_kernel + normalisation)", "bound": "tensor",
                     "achieved": achieved, "peak": peaks["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "flops": "executed: the symmetric X X^T and A A products run only their lower 256-tile "
                              "triangle (the value above counts the algorithmic 4 s^2 l + 2 s^3 per step)",
                     "frac": (achieved / peaks["bf16_tflops_sustained"]) if achieved else None,
                     "peak_source": f"bf16_tflops_sustained (cuBLAS bf16 under the power cap), {peak_src}",
                     "launches": n_n, "time_share": n_ms / ms if ms else None, "traffic": None},
        "gpu_launches": launches, "clocks": clk,
    }
    if not args.no_e2e:
        def e2e_step(xb, yb):
            _, b = step(xb, yb)
            return b, None
        ems = e2e_pipelined(e2e_step, gf, gd, args.steps, lambda: None, y_like=gd)
        out["e2e"] = {"value": fl * args.steps / (ems / 1000.0) / 1e12, "unit": "TFLOP/s",
                      "ms_per_step": ems / args.steps, "h2d_bytes_per_step": (gf.numel() + gd.numel()) * 4,
                      "d2h_bytes_per_step": gd.numel() * 4,
                      "path": "orthogonalize() on both gradients; every step copies them from pinned host memory "
                              "(side stream, double-buffered) and reads the down weight's update back"}
    if not args.no_cpu_baseline:
        from oracle import muon as om
        rng = np.random.default_rng(0)
        g1 = rng.standard_normal((1, d, h)).astype(np.float32)
        t0 = time.perf_counter()
        om.orthogonalize_f64(g1, om.coefficients(steps), dtype=np.float32)
        t1 = time.perf_counter() - t0
        est = 3 * t1  # the three slices have the same shape up to a transpose
        out["cpu_baseline"] = {"value": fl / est / 1e12, "unit": "TFLOP/s", "cores": cpu_cores(), "kind": "port",
                               "sample": f"the oracle's Newton-Schulz (numpy float32 BLAS on all host threads) on "
                                         f"one [{d}, {h}] slice, {steps} steps, times 3 slices",
                               "est_ms_per_step": est * 1000.0}
    return out


def run_layer(args, cfg, rank, world, local_rank, dev):
    """TransformerLayer(x, query_segment_ids=...) forward and the backward of its summed output; on
    N > 1 GPUs TransformerLayer(..., mesh=group): kv heads and GMLP hidden split, each rank holding
    B / N whole sequences."""
    import numpy as np
    import torch
    from macrogpt_jax_b200 import _capi, ops
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.layer import TransformerLayer
    from macrogpt_jax_b200.mlp import GMLP
    from macrogpt_jax_b200.soft_attn import SoftmaxAttention
    d, h, H, I, Dh, B, S = (cfg[k] for k in ("d", "h", "kv_heads", "group", "head_d", "B", "S"))
    if world > 1 and (B % world or H % world or h % world):
        raise SystemExit(f"the tensor-parallel layer needs batch {B}, kv heads {H} and hidden {h} divisible by {world}")
    T = B * S
    init = Einsum.override(initializer=scaled_normal_init(d ** -0.5))
    attn = SoftmaxAttention.override(kq_d=Dh, kv_heads=H, kv_q_ratio=I, q=init, k=init, v=init, o=init)
    mlp = GMLP.override(hidden_d=h, fused_proj=init, down_proj=Einsum.override(initializer=scaled_normal_init(h ** -0.5)))
    group = None
    if world > 1:
        import torch.distributed as dist
        group = dist.group.WORLD
    layer = TransformerLayer(d, attn=attn, mlp=mlp, rngs=Rngs(0), mesh=group)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234)
    x = torch.randn((B, S, d), generator=gen, device=dev).to(torch.bfloat16)
    dy = (torch.randn((B, S, d), generator=gen, device=dev) * 1e-3).to(torch.bfloat16)
    seg = torch.zeros((B, S), dtype=torch.int32, device=dev)
    if world > 1:  # this rank's whole sequences; segment ids stay full-batch
        bl = B // world
        x, dy = x[rank * bl:(rank + 1) * bl].contiguous(), dy[rank * bl:(rank + 1) * bl].contiguous()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())
    params = list(layer.parameters())

    def fwd_bwd(xb, dyb):
        xl = xb.detach().requires_grad_(True)
        y = layer(xl, query_segment_ids=seg)
        ev = torch.cuda.Event()
        ev.record()
        y.backward(dyb)
        for p in params:
            p.grad = None
        return y, ev

    for _ in range(args.warmup):
        fwd_bwd(x, dy)
    torch.cuda.synchronize()
    barrier()
    timer = ops.KernelTimer()
    clocks = ClockSampler(local_rank)
    clocks.start()
    launches0 = _capi.launches
    torch.cuda.synchronize()
    barrier()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ops.set_timer(timer)
    ev0.record()
    for _ in range(args.steps):
        fwd_bwd(x, dy)
    ev1.record()
    ops.set_timer(None)
    torch.cuda.synchronize()
    barrier()
    launches = _capi.launches - launches0
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    summ = timer.summary()
    peaks, peak_src = load_peaks()
    fl, proj_fl, attn_fl = layer_flops(cfg, T, S, B)
    g_n, g_ms, g_fl = summ.get("gemm", (0, 0.0, 0.0))
    peak_fp8 = 2.0 * peaks["bf16_tflops_sustained"]
    achieved = (g_fl / g_n) / (g_ms / g_n / 1000.0) / 1e12 if g_n else None
    out = {
        "metric": "FP8 Llama-3-8B transformer layer fwd+bwd tokens/s (TFLOP/s/GPU)",
        "value": T * args.steps / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp8", "data": "synthetic (seeded)",
        "config": {"workload": args.config_desc, "tokens": T, "d_model": d, "hidden": h, "q_heads": H * I,
                   "kv_heads": H, "head_dim": Dh,
                   "parallelism": "single GPU" if world == 1 else
                   f"tp{world} (kv heads of q/k/v/o and GMLP hidden split; token all-gather / reduce-scatter, "
                   f"B/{world} sequences per rank)",
                   "l2": "inputs larger than L2"},
        "tflops_per_gpu": fl * args.steps / (ms / 1000.0) / 1e12 / world,
        "flops_per_step": {"total": fl, "projections": proj_fl, "attention_causal": attn_fl,
                           "gmlp": 18.0 * T * d * h},
        "roofline": {"kernel": "gemm_fp8_pair_kernel (FP8 projections and GMLP)", "bound": "tensor",
                     "achieved": achieved, "peak": peak_fp8, "unit": "TFLOP/s",
                     "frac": (achieved / peak_fp8) if achieved else None,
                     "peak_source": f"2 x bf16_tflops_sustained, {peak_src}", "launches": g_n,
                     "time_share": g_ms / ms if ms else None, "traffic": None,
                     "note": "the attention's bf16 GEMMs are launched inside ufp8_attention_* and not in this record"},
        "gpu_launches": launches, "clocks": clk,
        "time_share": {k: round(v[1] / ms, 4) for k, v in summ.items()},
    }
    if not args.no_e2e:
        barrier()
        ems = max_over_ranks(e2e_pipelined(fwd_bwd, x, dy, args.steps, barrier))
        out["e2e"] = {"value": T * args.steps / (ems / 1000.0), "unit": "tokens/s", "ms_per_step": ems / args.steps,
                      "h2d_bytes_per_step": 2 * x.numel() * 2, "d2h_bytes_per_step": x.numel() * 2,
                      "path": "TransformerLayer forward + backward; x and dY in from pinned host memory each step "
                              "(side stream, double-buffered), y back (side stream, overlapping the backward)"}
    if rank != 0:
        return None
    if not args.no_cpu_baseline and world == 1:
        # The oracle's GMLP (hidden slice, full tokens) and attention (one kv-head group of one sequence)
        # timed and scaled by FLOPs; the projections at the GMLP port's FLOP rate.
        from oracle import attention as oa
        from oracle import path as op
        tg = cpu_oracle_step(d, 768, T, seed=0)
        rate = 18.0 * T * d * 768 / tg
        rng = np.random.default_rng(0)
        q = op.bf16_normal(rng, (1, S, I, Dh))
        k, v, go = op.bf16_normal(rng, (1, S, 1, Dh)), op.bf16_normal(rng, (1, S, 1, Dh)), op.bf16_normal(rng, (1, S, I, Dh))
        t0 = time.perf_counter()
        o, P = oa.attention_forward(q, k, v, scale=Dh ** -0.5)
        oa.attention_backward(go, o, P, q, k, v, Dh ** -0.5)
        ta = (time.perf_counter() - t0) * B * H
        est = 18.0 * T * d * h / rate + proj_fl / rate + ta
        out["cpu_baseline"] = {"value": T / est, "unit": "tokens/s", "cores": cpu_cores(), "kind": "port",
                               "sample": f"oracle GMLP at {T} tokens on a hidden slice of 768 (FLOP rate applied to the "
                                         f"GMLP and projection FLOPs) plus the oracle attention fwd+bwd of one kv-head "
                                         f"group of one {S}-token sequence times {B * H}",
                               "est_ms_per_step": est * 1000.0}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="gmlp_d4096")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--norm-unfused", action="store_true",
                    help="norm_gmlp_d4096: run RMSNorm and GMLP as separate modules (for comparison)")
    ap.add_argument("--no-tp-parity", action="store_true",
                    help="N > 1: skip the tensor-parallel vs single-GPU comparison printed as tp_parity")
    ap.add_argument("--gemm-traffic", type=float, default=None,
                    help="DRAM bytes per GEMM launch to report as roofline.traffic (default: the "
                         "captured figure for gmlp_d4096 on one GPU, else null)")
    ap.add_argument("--graph", action="store_true",
                    help="one GPU: capture the whole step in a CUDA graph and time its replays (for the "
                         "launch-bound small workloads)")
    ap.add_argument("--gemm-variant", type=int, default=0, choices=[0, 1, 2, 3],
                    help="GEMM kernel variant (ufp8_set_gemm_variant): 0 auto, 1 one CTA per tile, "
                         "2 CTA pair, 3 CTA pair with direct epilogue loads/stores")
    ap.add_argument("--tp-ag", choices=["sm", "ce"], default="ce",
                    help="P2P all-gather engine: an SM push kernel beside the GEMM, or copy engines")
    ap.add_argument("--tp-rs", choices=["p2p", "nccl"], default="p2p",
                    help="tensor-parallel collectives: NVLink P2P (all-gather and reduce-scatter with the GEMMs), "
                         "or NCCL")
    ap.add_argument("--tp-rs-engine", choices=["auto", "epilogue", "copy"], default="epilogue",
                    help="P2P reduce-scatter push: GEMM epilogue, copy engines beside independent work, or auto "
                         "(epilogue for y, copy engines for dx)")
    ap.add_argument("--tp-lanes", type=int, default=1, choices=range(1, 9),
                    help="streams the copy-engine pushes spread their per-peer copies over")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    cfg = CONFIGS[args.config]
    if cfg["kind"] == "attn":
        args.config_desc = (f"attention projections fwd+bwd (fused QKV {cfg['d']}->{3 * cfg['d']}, O "
                            f"{cfg['d']}->{cfg['d']}), {cfg['B'] * cfg['S']} tokens (B{cfg['B']} x S{cfg['S']}), "
                            f"{cfg['heads']} heads x {cfg['head_d']}, FP8 e4m3/e5m2")
        if args.impl == "reference":
            raise SystemExit("the CPU arm covers the GMLP workloads")
    elif cfg["kind"] == "layer":
        args.config_desc = (f"Llama-3-8B transformer layer fwd+bwd: RMSNorm -> FP8 q/k/v ({cfg['kv_heads'] * cfg['group']} "
                            f"query heads, {cfg['kv_heads']} kv heads x {cfg['head_d']}) -> RoPE -> causal softmax "
                            f"attention -> FP8 o, RMSNorm -> FP8 GMLP (h {cfg['h']}), {cfg['B'] * cfg['S']} tokens "
                            f"(B{cfg['B']} x S{cfg['S']})")
        if args.impl == "reference":
            raise SystemExit("the CPU arm covers the GMLP workloads")
    elif cfg["kind"] == "muon":
        args.config_desc = (f"Muon Newton-Schulz ({cfg['steps']} steps, coefficients 3.4445/-4.7750/2.0315) of a GMLP "
                            f"block's gradients: [2, {cfg['d']}, {cfg['h']}] and [{cfg['h']}, {cfg['d']}], f32 in/out, "
                            "bf16 GEMMs")
        if args.impl == "reference":
            raise SystemExit("the CPU arm covers the GMLP workloads")
    elif cfg["kind"] == "head":
        args.config_desc = (f"output head fwd+bwd (final RMSNorm -> FP8 lm_head {cfg['d']}->{cfg['V']} -> 15*tanh(l/15) "
                            f"-> next-token cross-entropy), {cfg['B'] * cfg['S']} tokens (B{cfg['B']} x S{cfg['S']}), "
                            "FP8 e4m3/e5m2")
    else:
        args.config_desc = (f"GMLP fwd+bwd, {cfg['B'] * cfg['S']} tokens (B{cfg['B']} x S{cfg['S']}), "
                            f"d_model {cfg['d']}, hidden {cfg['h']}, FP8 e4m3/e5m2")
        if cfg.get("norm"):
            args.config_desc = ("RMSNorm (uncentered) -> " + args.config_desc +
                                ("; norm and GMLP as separate modules" if args.norm_unfused else
                                 "; norm fused with the fp8 quantisation of its output"))
            if args.impl == "reference":
                raise SystemExit("the CPU arm covers the GMLP workloads")

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")

    # Libraries (NCCL's version banner, for one) write to file descriptor 1; send all of that
    # to stderr so that stdout carries exactly the one JSON line printed below.
    sys.stdout.flush()
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        out = run_reference(args, cfg, rank, world)
    else:
        if world > 1:
            import datetime
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                    device_id=torch.device("cuda", local_rank))
        try:
            out = run_ours(args, cfg, rank, world, local_rank)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
    if out is not None:
        print(json.dumps(out), file=json_out, flush=True)


if __name__ == "__main__":
    main()
