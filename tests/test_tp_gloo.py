"""Tensor-parallel GMLP host logic on CPU ranks (gloo, world size 2): weight slicing, global
per-tensor scales, fp8 all-gathers and token reduce-scatters, checked against the
single-device oracle; plus the failure paths (mismatched sizes, a rank that never joins)."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

T, D, H = 64, 32, 64


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir):
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from cpu_backend import CpuBackend
    from macrogpt_jax_b200.einsum import Rngs, scaled_normal_init
    from macrogpt_jax_b200.tp import TPGMLP
    from oracle import path as op
    m = TPGMLP(D, H, rngs=Rngs(5), device=torch.device("cpu"), fused_init=scaled_normal_init(D ** -0.5),
               down_init=scaled_normal_init(H ** -0.5), backend=CpuBackend())
    rng = np.random.default_rng(0)  # identical full activations on every rank
    xb = op.bf16_normal(rng, (T, D))
    dyb = op.bf16_normal(rng, (T, D), 1e-3)
    to_t = lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    x = m.shard_tokens(to_t(xb)).requires_grad_(True)
    y = m(x)
    y.backward(m.shard_tokens(to_t(dyb)))
    bits = lambda t: t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), y=bits(y), dx=bits(x.grad), dwf=bits(m.fused_proj.w.grad),
             dwd=bits(m.down_proj.w.grad), wf=bits(m.fused_proj.w), wd=bits(m.down_proj.w))
    dist.destroy_process_group()


def test_tp2_matches_single_device_oracle(tmp_path):
    from helpers import bf16_bits_to_f64, compare
    from macrogpt_jax_b200.einsum import Rngs, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP
    from macrogpt_jax_b200.einsum import Einsum
    from oracle import path as op
    mp.spawn(_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]
    full = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(D ** -0.5)),
                         down_proj=Einsum.override(initializer=scaled_normal_init(H ** -0.5)))(
        D, H, rngs=Rngs(5))
    bits = lambda t: t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    wf, wd = bits(full.fused_proj.w), bits(full.down_proj.w)
    # the shards are exact slices of the single-device weights
    assert (np.concatenate([r[0]["wf"], r[1]["wf"]], axis=2) == wf).all()
    assert (np.concatenate([r[0]["wd"], r[1]["wd"]], axis=0) == wd).all()
    rng = np.random.default_rng(0)
    xb = op.bf16_normal(rng, (T, D))
    dyb = op.bf16_normal(rng, (T, D), 1e-3)
    y, saved = op.gmlp_forward(xb, wf, wd)
    g = op.gmlp_backward(dyb, saved)
    f = bf16_bits_to_f64
    compare(f(np.concatenate([r[0]["y"], r[1]["y"]])), f(y))
    compare(f(np.concatenate([r[0]["dx"], r[1]["dx"]])), f(g["dx"]))
    compare(f(np.concatenate([r[0]["dwf"], r[1]["dwf"]], axis=2)), f(g["dwf"]))
    compare(f(np.concatenate([r[0]["dwd"], r[1]["dwd"]], axis=0)), f(g["dwd"]))


def _bad_hidden(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    from macrogpt_jax_b200.einsum import Rngs
    from macrogpt_jax_b200.tp import TPGMLP
    try:
        with pytest.raises(ValueError, match="not divisible"):
            TPGMLP(8, 31, rngs=Rngs(0), device=torch.device("cpu"))
    finally:
        dist.destroy_process_group()


def test_tp_rejects_indivisible_hidden():
    mp.spawn(_bad_hidden, args=(2, _port()), nprocs=2, join=True)


def _lonely(rank, world, port, q):
    """Rank 0 of a 2-rank group whose peer never joins: the short rendezvous timeout turns
    the missing rank into an error on the host instead of a hang."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_missing_rank_fails_fast():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(0, 2, _port(), q))
    p.start()
    p.join(60)
    assert not p.is_alive()
    assert q.get(timeout=5) != "joined"


def _mesh_worker(rank, world, port, outdir):
    """The reference's own drop-in: GMLP.override(...)(..., mesh=<tensor group>) builds the
    tensor-parallel block; and Einsum.reshard(mesh) slices a weight along its 'tensor' axis."""
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from cpu_backend import CpuBackend
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP
    from oracle import path as op
    group = dist.new_group(list(range(world)))
    m = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(D ** -0.5)),
                      down_proj=Einsum.override(initializer=scaled_normal_init(H ** -0.5)))(
        D, H, rngs=Rngs(5), mesh=group, tp_backend=CpuBackend())
    assert tuple(m.fused_proj.w.shape) == (2, D, H // world) and tuple(m.down_proj.w.shape) == (H // world, D)
    rng = np.random.default_rng(0)
    xb = op.bf16_normal(rng, (T, D))
    dyb = op.bf16_normal(rng, (T, D), 1e-3)
    to_t = lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    x = m.shard_tokens(to_t(xb)).requires_grad_(True)
    y = m(x)
    y.backward(m.shard_tokens(to_t(dyb)))
    bits = lambda t: t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    e = Einsum("bnd,dh->bnh", initializer=scaled_normal_init(0.1), size_dict={"d": D, "h": H}, rngs=Rngs(9),
               sharding=(None, "tensor"), device=torch.device("cpu"))
    full_e = bits(e.w)
    e.reshard(group)
    assert e.shard == (1, rank, world) and e.size_dict["h"] == H // world
    assert e.metadata.canonical_shape == (D, H // world)
    np.savez(os.path.join(outdir, f"mesh{rank}.npz"), y=bits(y), dx=bits(x.grad), dwf=bits(m.fused_proj.w.grad),
             dwd=bits(m.down_proj.w.grad), e_full=full_e, e_local=bits(e.w))
    dist.destroy_process_group()


def test_gmlp_with_mesh_is_tensor_parallel(tmp_path):
    from helpers import bf16_bits_to_f64, compare
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP
    from oracle import path as op
    mp.spawn(_mesh_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"mesh{i}.npz") for i in range(2)]
    full = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(D ** -0.5)),
                         down_proj=Einsum.override(initializer=scaled_normal_init(H ** -0.5)))(
        D, H, rngs=Rngs(5))
    bits = lambda t: t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    wf, wd = bits(full.fused_proj.w), bits(full.down_proj.w)
    rng = np.random.default_rng(0)
    xb = op.bf16_normal(rng, (T, D))
    dyb = op.bf16_normal(rng, (T, D), 1e-3)
    y, saved = op.gmlp_forward(xb, wf, wd)
    g = op.gmlp_backward(dyb, saved)
    f = bf16_bits_to_f64
    compare(f(np.concatenate([r[0]["y"], r[1]["y"]])), f(y))
    compare(f(np.concatenate([r[0]["dx"], r[1]["dx"]])), f(g["dx"]))
    compare(f(np.concatenate([r[0]["dwf"], r[1]["dwf"]], axis=2)), f(g["dwf"]))
    compare(f(np.concatenate([r[0]["dwd"], r[1]["dwd"]], axis=0)), f(g["dwd"]))
    # reshard: each rank holds its contiguous column block of the same full weight
    assert (r[0]["e_full"] == r[1]["e_full"]).all()
    assert (np.concatenate([r[0]["e_local"], r[1]["e_local"]], axis=1) == r[0]["e_full"]).all()


def _rows_worker(rank, world, port, outdir):
    """gather_rows / scatter_rows (the token all-gather and reduce-scatter the tensor-parallel
    attention wraps around its local heads) and their gradients, on CPU ranks."""
    import sys
    sys.path.insert(0, os.path.dirname(__file__))
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    from cpu_backend import CpuBackend
    from macrogpt_jax_b200.tp import TPContext, gather_rows, scatter_rows
    tp = TPContext(backend=CpuBackend())
    assert not tp.fused_rs
    gen = torch.Generator().manual_seed(100 + rank)
    x = torch.randn((3, 2, 5), generator=gen, dtype=torch.float64).requires_grad_(True)
    c = float(rank + 2)
    full = gather_rows(x, tp)
    y = scatter_rows(full * c, tp)
    g = torch.randn(y.shape, generator=gen, dtype=torch.float64)
    y.backward(g)
    np.savez(os.path.join(outdir, f"rows{rank}.npz"), x=x.detach().numpy(), full=full.detach().numpy(),
             y=y.detach().numpy(), g=g.numpy(), dx=x.grad.numpy())
    dist.destroy_process_group()


def test_gather_scatter_rows_autograd(tmp_path):
    """y_r = block r of sum_s c_s * cat(x) = (c_0 + c_1) x_r, and dx_r = (c_0 + c_1) g_r."""
    mp.spawn(_rows_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"rows{i}.npz") for i in range(2)]
    cat = np.concatenate([r[0]["x"], r[1]["x"]])
    for i in range(2):
        np.testing.assert_array_equal(r[i]["full"], cat)
        np.testing.assert_allclose(r[i]["y"], 5.0 * r[i]["x"], rtol=1e-12)
        np.testing.assert_allclose(r[i]["dx"], 5.0 * r[i]["g"], rtol=1e-12)
