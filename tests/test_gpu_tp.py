"""Tensor-parallel FP8 GMLP on 2 GPUs (NCCL, one process per GPU) against the oracle.
Skips when fewer than two GPUs are visible."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

T, D, H = 512, 256, 1024


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, outdir, fused=True, ag_engine=1, rs_engine="auto", lanes=2):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from macrogpt_jax_b200 import tp as tp_mod
        from macrogpt_jax_b200.einsum import Rngs, scaled_normal_init
        from macrogpt_jax_b200.tp import TPGMLP
        tp_mod.AG_ENGINE = ag_engine
        tp_mod.RS_ENGINE = rs_engine
        tp_mod.COPY_LANES = lanes
        from oracle import path as op
        dev = torch.device("cuda", rank)
        m = TPGMLP(D, H, rngs=Rngs(7), device=dev, fused_init=scaled_normal_init(D ** -0.5),
                   down_init=scaled_normal_init(H ** -0.5), fused_reduce_scatter=fused)
        assert m.tp.fused_rs == fused
        rng = np.random.default_rng(0)
        xb = op.bf16_normal(rng, (T, D))
        dyb = op.bf16_normal(rng, (T, D), 1e-3)
        to_t = lambda b: torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(dev)  # noqa: E731
        bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        first = None
        for it in range(3):  # every staging buffer used at least twice: results must repeat bit for bit
            for p in m.parameters():
                p.grad = None
            x = m.shard_tokens(to_t(xb)).requires_grad_(True)
            y = m(x)
            y.backward(m.shard_tokens(to_t(dyb)))
            torch.cuda.synchronize()
            now = [bits(t) for t in (y, x.grad, m.fused_proj.w.grad, m.down_proj.w.grad)]
            if first is None:
                first = now
            else:
                assert all(np.array_equal(a, b) for a, b in zip(first, now)), f"iteration {it} differs"
        from macrogpt_jax_b200 import _capi
        assert _capi.device_status() == 0
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), y=bits(y), dx=bits(x.grad),
                 dwf=bits(m.fused_proj.w.grad), dwd=bits(m.down_proj.w.grad))
        m.tp.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fused,ag_engine,rs_engine,lanes",
                         [(True, 1, "epilogue", 1), (True, 0, "epilogue", 1), (True, 0, "auto", 2),
                          (True, 0, "copy", 3), (False, 1, "auto", 2)],
                         ids=["p2p_sm_push", "p2p_copy_engine", "p2p_auto_2lanes", "p2p_copy_rs_3lanes", "nccl"])
def test_tp2_gpu_matches_oracle(cuda, tmp_path, fused, ag_engine, rs_engine, lanes):
    """All-gather by SM push kernel or copy engines (1..3 lanes), reduce-scatter pushed from the
    GEMM epilogue, by copy engines, or auto (epilogue for y, copy engines beside dWf for dx)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from helpers import bf16_bits_to_f64, compare
    from macrogpt_jax_b200.einsum import Einsum, Rngs, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP
    from oracle import path as op
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_worker, args=(2, _port(), str(tmp_path), fused, ag_engine, rs_engine, lanes), nprocs=2, join=True)
    r = [np.load(tmp_path / f"rank{i}.npz") for i in range(2)]
    cpu = torch.device("cpu")
    full = GMLP.override(fused_proj=Einsum.override(initializer=scaled_normal_init(D ** -0.5), device=cpu),
                         down_proj=Einsum.override(initializer=scaled_normal_init(H ** -0.5), device=cpu))(
        D, H, rngs=Rngs(7))
    bits = lambda t: t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    rng = np.random.default_rng(0)
    xb = op.bf16_normal(rng, (T, D))
    dyb = op.bf16_normal(rng, (T, D), 1e-3)
    y, saved = op.gmlp_forward(xb, bits(full.fused_proj.w), bits(full.down_proj.w))
    g = op.gmlp_backward(dyb, saved)
    f = bf16_bits_to_f64
    compare(f(np.concatenate([r[0]["y"], r[1]["y"]])), f(y))
    compare(f(np.concatenate([r[0]["dx"], r[1]["dx"]])), f(g["dx"]))
    compare(f(np.concatenate([r[0]["dwf"], r[1]["dwf"]], axis=2)), f(g["dwf"]))
    compare(f(np.concatenate([r[0]["dwd"], r[1]["dwd"]], axis=0)), f(g["dwd"]))


DA, SA, BA, KV = 256, 256, 4, 4  # attention block: model width, sequence, batch, kv heads


def _attn_factories():
    from macrogpt_jax_b200.einsum import Einsum, scaled_normal_init
    from macrogpt_jax_b200.mlp import GMLP
    from macrogpt_jax_b200.soft_attn import SoftmaxAttention
    init = Einsum.override(initializer=scaled_normal_init(DA ** -0.5))
    attn = SoftmaxAttention.override(kq_d=64, kv_heads=KV, kv_q_ratio=2, q=init, k=init, v=init, o=init)
    mlp = GMLP.override(hidden_d=4 * DA, fused_proj=init, down_proj=Einsum.override(
        initializer=scaled_normal_init((4 * DA) ** -0.5)))
    return attn, mlp


def _attn_inputs(dev):
    rng = np.random.default_rng(21)
    x = torch.from_numpy(rng.standard_normal((BA, SA, DA)).astype(np.float32)).to(torch.bfloat16).to(dev)
    dy = torch.from_numpy(rng.standard_normal((BA, SA, DA)).astype(np.float32) * 1e-2).to(torch.bfloat16).to(dev)
    seg = torch.zeros((BA, SA), dtype=torch.int32, device=dev)
    seg[1, SA // 3:] = 1
    seg[3, SA - 40:] = -1
    return x, dy, seg


def _layer_parts(layer, seg):
    """The whole layer (full-batch ids) and its two residual branches alone."""
    from macrogpt_jax_b200.layer import norm_mlp
    return {"l": lambda z: layer(z, query_segment_ids=seg),
            "la": lambda z: z + layer.attn(layer.attn_norm(z), None, query_segment_ids=seg),
            "lm": lambda z: z + norm_mlp(layer.mlp_norm, layer.mlp, z)}


def _attn_worker(rank, world, port, outdir):
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(__file__)))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from macrogpt_jax_b200.einsum import Rngs
        from macrogpt_jax_b200.layer import TransformerLayer
        attn_f, mlp_f = _attn_factories()
        group = dist.group.WORLD
        x, dy, seg = _attn_inputs(dev)
        bl = BA // world
        sl = slice(rank * bl, (rank + 1) * bl)
        bits = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
        out = {}
        a = attn_f(model_d=DA, rngs=Rngs(3), mesh=group)
        assert a.kv_heads == KV // world and a.q.w.shape[1] == KV // world
        xl = x[sl].clone().requires_grad_(True)
        y = a(xl, query_segment_ids=seg[sl])  # local ids, gathered inside
        y.backward(dy[sl])
        out.update(a_y=bits(y), a_dx=bits(xl.grad), a_dq=bits(a.q.w.grad), a_dk=bits(a.k.w.grad),
                   a_dv=bits(a.v.w.grad), a_do=bits(a.o.w.grad))
        layer = TransformerLayer(DA, attn=attn_f, mlp=mlp_f, rngs=Rngs(4), mesh=group)
        for key, fn in _layer_parts(layer, seg).items():
            xl = x[sl].clone().requires_grad_(True)
            y = fn(xl)
            y.backward(dy[sl])
            out.update({f"{key}_y": bits(y), f"{key}_dx": bits(xl.grad)})
        out.update(l_dwd=bits(layer.mlp.down_proj.w.grad), l_do=bits(layer.attn.o.w.grad))
        torch.cuda.synchronize()
        from macrogpt_jax_b200 import _capi
        assert _capi.device_status() == 0
        np.savez(os.path.join(outdir, f"attn{rank}.npz"), **out)
        a._tp.close()
        layer.attn._tp.close()
        layer.mlp._tp.tp.close()
    finally:
        dist.destroy_process_group()


def test_tp2_attention_and_layer_match_single_gpu(cuda, tmp_path):
    """SoftmaxAttention(mesh=group) (kv heads split, token all-gather / reduce-scatter) and a
    TransformerLayer(mesh=group) (that attention + the tensor-parallel GMLP) on 2 GPUs against
    the same modules on one GPU built from the same seed: outputs, input gradients and the
    weight-gradient shards of the attention, and each residual branch of the layer, at the GEMM
    bar.  The whole layer is held to rel 0.1 / cosine 0.999: its MLP quantises the attention
    branch's output, whose bf16 sums differ in order between the two runs, and an input that
    moves by one bf16 step can round to a neighbouring fp8 value (2^-3 relative for e4m3), which
    the MLP then carries forward."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    from helpers import compare
    from macrogpt_jax_b200.einsum import Rngs
    from macrogpt_jax_b200.layer import TransformerLayer
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    mp.spawn(_attn_worker, args=(2, _port(), str(tmp_path)), nprocs=2, join=True)
    r = [np.load(tmp_path / f"attn{i}.npz") for i in range(2)]
    attn_f, mlp_f = _attn_factories()
    x, dy, seg = _attn_inputs(cuda)
    a = attn_f(model_d=DA, rngs=Rngs(3))
    xg = x.clone().requires_grad_(True)
    y = a(xg, query_segment_ids=seg)
    y.backward(dy)
    f = lambda t: t.detach().double().cpu().numpy()  # noqa: E731
    cat = lambda key, axis=0: np.concatenate([r[0][key], r[1][key]], axis=axis).astype(np.float64)  # noqa: E731
    compare(cat("a_y"), f(y))
    compare(cat("a_dx"), f(xg.grad))
    compare(cat("a_dq", 1), f(a.q.w.grad))
    compare(cat("a_dk", 1), f(a.k.w.grad))
    compare(cat("a_dv", 1), f(a.v.w.grad))
    compare(cat("a_do", 0), f(a.o.w.grad))
    layer = TransformerLayer(DA, attn=attn_f, mlp=mlp_f, rngs=Rngs(4))
    for key, fn in _layer_parts(layer, seg).items():
        xg = x.clone().requires_grad_(True)
        y = fn(xg)
        y.backward(dy)
        bar = dict(rel_tol=0.1, cos_tol=0.999) if key == "l" else {}
        compare(cat(f"{key}_y"), f(y), **bar)
        compare(cat(f"{key}_dx"), f(xg.grad), **bar)
    # weight gradients accumulated over the three passes (whole layer and both branches)
    compare(cat("l_dwd", 0), f(layer.mlp.down_proj.w.grad), rel_tol=0.1, cos_tol=0.999)
    compare(cat("l_do", 0), f(layer.attn.o.w.grad), rel_tol=0.1, cos_tol=0.999)
