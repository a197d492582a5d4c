"""Reduce-scatter contexts on one GPU: the RS_PUSH epilogue + finish data path (world size 1)
and the failure path — a peer that never signals makes the bounded wait run out and report
UFP8_STATUS_PEER_TIMEOUT instead of hanging.  No kernel here waits on another kernel."""
import time

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("variant", [0, 3], ids=["staged", "direct"])
@pytest.mark.parametrize("d", [256, 208], ids=["d256", "ragged_cols"])
def test_rs_push_world1_matches_store(cuda, variant, d):
    """F2 with the RS_PUSH epilogue into a one-rank staging slot, then finish: bit-identical
    to the plain-store epilogue (one slot summed in fp32 is exact).  Covers the staged
    (bulk-store) and direct kernels and a ragged last column block (208 = 3 x 64 + 16, whose
    last 16 columns take the plain-store fallback)."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    C.set_gemm_variant(variant)
    T, h = 512, 384
    gen = torch.Generator(device=cuda)
    gen.manual_seed(3)
    qh = ops.quantize(torch.randn((T, h), generator=gen, device=cuda).to(torch.bfloat16), C.E4M3)
    qwd = ops.quantize((torch.randn((h, d), generator=gen, device=cuda) * 0.05).to(torch.bfloat16), C.E4M3)
    y_ref = ops.gmlp_f2(qh, qwd)
    rs = C.TPReduceScatter(0, 1, ((T * d * 2 + 255) // 256) * 256)
    rs.connect([rs.handle])
    try:
        for _ in range(3):  # both staging buffers, then reuse
            table, epoch = rs.begin()
            ops.gmlp_f2_push(qh, qwd, table, 0, T)
            out = torch.empty(T, d, dtype=torch.bfloat16, device=cuda)
            rs.finish(epoch, T, d, d, out.data_ptr(), d, torch.cuda.current_stream().cuda_stream)
            torch.cuda.synchronize()
            assert torch.equal(out, y_ref)
        assert C.device_status() == 0
    finally:
        rs.close()
        C.set_gemm_variant(0)


def test_missing_peer_times_out(cuda):
    """Rank 0 of a two-rank group whose rank 1 never finishes: rank 0's finish gives up after
    its 200 ms limit, sets the peer-timeout status bit, and the GPU stays usable."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    rows, cols = 64, 64
    a = C.TPReduceScatter(0, 2, rows * cols * 2)
    b = C.TPReduceScatter(1, 2, rows * cols * 2)
    a.connect_local([a, b])
    b.connect_local([a, b])
    a.set_timeout_ms(200)
    _, epoch = a.begin()
    out = torch.zeros(rows, cols, dtype=torch.bfloat16, device=cuda)
    t0 = time.time()
    a.finish(epoch, rows, cols, cols, out.data_ptr(), cols, torch.cuda.current_stream().cuda_stream)
    status = C.device_status(clear=True)
    assert status & C.STATUS_PEER_TIMEOUT
    assert time.time() - t0 < 10
    assert C.device_status() == 0
    x = torch.ones(10, device=cuda)
    assert float((x * 2).sum()) == 20.0
    a.close()
    b.close()


def test_unconnected_context_is_refused(cuda):
    from macrogpt_jax_b200 import _capi as C
    a = C.TPReduceScatter(0, 2, 256)
    with pytest.raises(C.UFP8Error, match="not connected"):
        a.begin()
    a.close()


def test_allreduce_max_world1_and_nan(cuda):
    """The P2P MAX exchange of a one-rank group returns its input, NaN included, bit for bit."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    ex = C.TPReduceScatter(0, 1, 256)
    ex.connect([ex.handle])
    try:
        stream = torch.cuda.current_stream().cuda_stream
        for vals in ([3.5], [0.0, 448.0, 1e-30], [1.0, float("nan"), float("inf"), 2.0, 0.5, 7.0, 8.0, 9.0]):
            a = torch.tensor(vals, dtype=torch.float32, device=cuda)
            out = torch.full_like(a, -1.0)
            ex.allreduce_max(a.data_ptr(), out.data_ptr(), a.numel(), stream)
            torch.cuda.synchronize()
            assert torch.equal(out.view(torch.int32), a.view(torch.int32))
        with pytest.raises(C.UFP8Error, match="n = 9"):
            ex.allreduce_max(a.data_ptr(), out.data_ptr(), 9, stream)
        assert C.device_status() == 0
    finally:
        ex.close()


def test_allreduce_max_missing_peer_times_out(cuda):
    """Rank 0 of a two-rank group whose rank 1 never calls: the exchange gives up after its
    200 ms limit, sets the peer-timeout bit, leaves `out` unchanged, and the GPU stays usable."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    a = C.TPReduceScatter(0, 2, 256)
    b = C.TPReduceScatter(1, 2, 256)
    a.connect_local([a, b])
    b.connect_local([a, b])
    a.set_timeout_ms(200)
    try:
        x = torch.tensor([1.0, 2.0], device=cuda)
        out = torch.full_like(x, -1.0)
        a.allreduce_max(x.data_ptr(), out.data_ptr(), 2, torch.cuda.current_stream().cuda_stream)
        assert C.device_status(clear=True) & C.STATUS_PEER_TIMEOUT
        assert torch.equal(out.cpu(), torch.tensor([-1.0, -1.0]))
        assert C.device_status() == 0
    finally:
        a.close()
        b.close()


def _ag_setup(cuda, world, rows_per_rank, d):
    """A connected group of `world` contexts on this GPU; returns rank 0's context, epoch and
    its arrival flags as an int32 tensor view."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200.tp import _device_bytes
    ctxs = [C.TPReduceScatter(r, world, rows_per_rank * d) for r in range(world)]
    for c in ctxs:
        c.connect_local(ctxs)
    _, epoch = ctxs[0].begin()
    _, flags_ptr = ctxs[0].local(epoch)
    flags = _device_bytes(flags_ptr, (4 * world,), cuda).view(torch.int32)
    return ctxs, epoch, flags_ptr, flags


@pytest.mark.parametrize("ag_rank", [0, 2])
def test_all_gathered_f1_matches_plain(cuda, ag_rank):
    """F1 whose x row blocks are marked arrived through the all-gather flags (tile order
    rotated to this rank's block, one block per raster group) equals the plain F1 bit for bit."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    world, rl, d, h = 4, 256, 256, 384
    gen = torch.Generator(device=cuda)
    gen.manual_seed(5)
    qx = ops.quantize(torch.randn((world * rl, d), generator=gen, device=cuda).to(torch.bfloat16), C.E4M3)
    qwf = ops.quantize((torch.randn((2, d, h), generator=gen, device=cuda) * 0.06).to(torch.bfloat16), C.E4M3)
    ref = ops.gmlp_f1(qx, qwf)
    ctxs, epoch, flags_ptr, flags = _ag_setup(cuda, world, rl, d)
    try:
        flags.fill_(epoch)
        got = ops.gmlp_f1(qx, qwf, ag=(flags_ptr, epoch, ag_rank, rl))
        torch.cuda.synchronize()
        for a, b in zip(got, ref):
            assert torch.equal(a, b)
        assert C.device_status() == 0
    finally:
        for c in ctxs:
            c.close()


def test_all_gather_missing_block_times_out(cuda):
    """A row block whose arrival flag nothing sets: the GEMM producer gives up after its bounded
    wait, the peer-timeout bit is set and the GPU stays usable."""
    import torch
    from macrogpt_jax_b200 import _capi as C
    from macrogpt_jax_b200 import ops
    world, rl, d, h = 2, 256, 128, 128
    qx = ops.quantize(torch.ones((world * rl, d), dtype=torch.bfloat16, device=cuda), C.E4M3)
    qwf = ops.quantize(torch.ones((2, d, h), dtype=torch.bfloat16, device=cuda), C.E4M3)
    ctxs, epoch, flags_ptr, flags = _ag_setup(cuda, world, rl, d)
    try:
        flags.zero_()
        t0 = time.time()
        ops.gmlp_f1(qx, qwf, ag=(flags_ptr, epoch, 0, rl))
        status = C.device_status(clear=True)
        assert status & C.STATUS_PEER_TIMEOUT
        assert time.time() - t0 < 30
        assert C.device_status() == 0
        assert float((torch.ones(8, device=cuda) * 3).sum()) == 24.0
    finally:
        for c in ctxs:
            c.close()
