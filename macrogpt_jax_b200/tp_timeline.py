"""Kernel timeline of one tensor-parallel GMLP step on every GPU of a node (torch.profiler).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \\
        -m macrogpt_jax_b200.tp_timeline [--tp-rs p2p|nccl] [--tp-ag ce|sm] [--tp-lanes N]
        [--tp-rs-engine auto|epilogue|copy] [--out DIR]

Builds the TPGMLP of the tensor-parallel bench workload (16384 tokens, d_model 4096, hidden
14336), runs 5 untimed steps, then records 3 steps with torch.profiler (CUDA activity only) and
writes, for the first and the last rank, one line per GPU activity (kernels, peer copies,
memsets): start offset in us from the first recorded activity, duration in us, stream, name.
Timestamps come from CUPTI on the host clock, so the ranks' files line up to a few us.
"""
from __future__ import annotations

import argparse
import datetime
import os

import torch
import torch.distributed as dist


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--tp-rs", choices=["p2p", "nccl"], default="p2p")
    ap.add_argument("--tp-ag", choices=["ce", "sm"], default="ce")
    ap.add_argument("--tp-lanes", type=int, default=1)
    ap.add_argument("--tp-rs-engine", choices=["auto", "epilogue", "copy"], default="epilogue")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=14336)
    ap.add_argument("--out", default="timelines")
    args = ap.parse_args()

    from torch.profiler import ProfilerActivity, profile

    from . import _capi as C
    from . import tp as tp_mod
    from .einsum import Rngs, scaled_normal_init

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    try:
        tp_mod.AG_ENGINE = C.AG_COPY_ENGINE if args.tp_ag == "ce" else C.AG_SM
        tp_mod.COPY_LANES = args.tp_lanes
        tp_mod.RS_ENGINE = args.tp_rs_engine
        d, h, T = args.d, args.hidden, args.tokens
        mlp = tp_mod.TPGMLP(model_d=d, hidden_d=h, rngs=Rngs(0), device=dev,
                            fused_init=scaled_normal_init(d ** -0.5), down_init=scaled_normal_init(h ** -0.5),
                            fused_reduce_scatter=args.tp_rs == "p2p")
        gen = torch.Generator(device=dev)
        gen.manual_seed(1)
        x = torch.randn((T // world, d), generator=gen, device=dev).to(torch.bfloat16)
        dy = (torch.randn((T // world, d), generator=gen, device=dev) * 1e-3).to(torch.bfloat16)
        params = list(mlp.parameters())

        def step():
            xl = x.detach().requires_grad_(True)
            mlp(xl).backward(dy)
            for p in params:
                p.grad = None

        for _ in range(5):
            step()
        torch.cuda.synchronize()
        dist.barrier()
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            for _ in range(3):
                step()
            torch.cuda.synchronize()
        dist.barrier()
        if rank in (0, world - 1):
            evs = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
                         key=lambda e: e.time_range.start)
            t0 = evs[0].time_range.start if evs else 0.0
            os.makedirs(args.out, exist_ok=True)
            path = os.path.join(args.out, f"timeline_tp{world}_{args.tp_rs}_{args.tp_ag}{args.tp_lanes}_{args.tp_rs_engine}_rank{rank}.txt")
            with open(path, "w") as f:
                for e in evs:
                    f.write(f"{e.time_range.start - t0:10.1f} {e.time_range.elapsed_us():8.1f} "
                            f"s{getattr(e, 'device_resource_id', '?')} {e.name[:90]}\n")
        mlp.tp.close()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
