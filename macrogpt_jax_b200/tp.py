"""Tensor-parallel FP8 GMLP across the GPUs of one box (one process per GPU).

The reference declares this split but never builds a mesh (ueaj/model/mlp.py:85,96 put
'tensor' on the hidden axis of both weights; ueaj/model/layer.py:9,57 shard activations over
tokens).  Here it runs for real:

  * gate/up weight column-split over hidden: rank r holds Wf[:, :, r*h/k:(r+1)*h/k], so
    swish(gate) * up stays local; down weight row-split: Wd[r*h/k:(r+1)*h/k, :];
  * activations are token-sharded [T/k, d] between blocks;
  * forward: all-gather fp8 x -> local [U, G, H] GEMM -> local partial y = H Wd over this
    rank's hidden slice -> reduce-scatter of the partials over tokens;
  * backward mirrors it: all-gather fp8 dY -> local dH/gating and dWd -> local partial dx
    -> reduce-scatter; dWf and dWd stay local (no data-parallel all-reduce in this block).

Every per-tensor scale is the scale of the WHOLE logical tensor (a MAX all-reduce of the
local amax values), so each rank quantises exactly as the single-GPU path does; the only
numerical difference from one GPU is the order of the final bf16 sums.

With the CUDA backend (default) every collective of the step runs over NVLink peer memory
through this package's C ABI (see TPContext): the all-gathers are copy-engine pushes consumed
block by block by the next GEMM, the reduce-scatters are pushed from the GEMM epilogues, and
the amax MAX all-reduces are single-warp exchanges.  With `fused_reduce_scatter=False`, or a
substituted backend (the tests use a CPU backend to exercise the host logic over gloo), they
go through torch.distributed instead (NCCL on GPUs).
"""
from __future__ import annotations

import warnings
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _capi as C
from . import ops as cuda_ops
from .configurator import config
from .einsum import Einsum, Rngs, lecun_normal_init, zeros_init


# How the all-gather moves each rank's block to its peers: C.AG_COPY_ENGINE (cudaMemcpyAsync
# per peer, no SM resources) or C.AG_SM (a small push kernel).  The copy engines win at TP 8:
# the push kernel's CTAs hold the SMs that the consuming GEMM (one CTA pair per two SMs with
# ~225 KiB of shared memory each) needs, so the GEMM starts only when the push ends.
AG_ENGINE = C.AG_COPY_ENGINE

# Streams over which the copy-engine pushes spread their per-peer copies (ufp8_tp_set_copy_lanes).
# Measured at TP 4 (GMLP, 16384 tokens, d 4096, h 14336): 2 lanes 2.27 ms/step and 3 lanes 3.14
# against 2.21 with 1 (copy engines running at once slow each other down), so 1 is the default.
COPY_LANES = 1

# How each reduce-scatter's partial rows reach their owners: "epilogue" (the GEMM epilogue
# stores them into the peers' slots, UFP8_EPI_RS_PUSH), "copy" (the GEMM stores locally and
# copy engines push the blocks, ufp8_tp_rs_push_copy, while independent work runs), or "auto":
# the epilogue push for y (nothing in the forward can run beside it) and copy engines for dx
# (dWf = x^T dUG runs while the blocks travel).  "auto" wins at TP 2 (4.00 vs 4.08 ms/step) and
# loses badly at TP 4 (3.94 vs 2.21), so the epilogue push is the default.
RS_ENGINE = "epilogue"


def tensor_group(mesh):
    """The process group of the 'tensor' axis of `mesh` (ueaj/model/mlp.py:85,96 and
    ueaj/model/einsum.py:218-220 shard weights over that axis), or None when there is no such
    axis or it has a single rank.  `mesh` may be a torch DeviceMesh with a dimension named
    'tensor' or a ProcessGroup (taken as the tensor axis); anything else (None, or a mesh
    description this package does not run on, which layers only record) has no tensor axis."""
    if mesh is None or not dist.is_available() or not dist.is_initialized():
        return None
    if hasattr(mesh, "mesh_dim_names") and hasattr(mesh, "get_group"):
        names = tuple(mesh.mesh_dim_names or ())
        if "tensor" not in names:
            return None
        group = mesh.get_group("tensor")
    elif isinstance(mesh, dist.ProcessGroup):
        group = mesh
    else:
        return None
    return group if dist.get_world_size(group) > 1 else None


class _DeviceBytes:
    """A raw device allocation seen through __cuda_array_interface__ (no ownership)."""

    def __init__(self, ptr: int, shape):
        self.__cuda_array_interface__ = {"data": (ptr, False), "shape": tuple(shape), "typestr": "|u1",
                                         "strides": None, "version": 3}


def _device_bytes(ptr: int, shape, device) -> torch.Tensor:
    return torch.as_tensor(_DeviceBytes(ptr, shape), device=device)


class TPContext:
    """Process group, rank layout and compute backend of one tensor-parallel block.

    With the CUDA backend and `fused_reduce_scatter` the reduce-scatters run over NVLink peer
    memory: the down-projection / dx GEMM epilogues store each partial row straight into its
    owner's staging slot (UFP8_EPI_RS_PUSH) and ufp8_tp_finish sums the slots on the owner,
    so the transfer overlaps the GEMM tile by tile; the MAX all-reduces of the amax values
    are then single-warp P2P exchanges (ufp8_tp_allreduce_max) instead of NCCL calls.
    Otherwise NCCL's reduce-scatter runs after the GEMM and NCCL all-reduces the amax values.

    Construction is collective.  With the P2P path it connects the exchange context right away
    and the ranks agree (a MIN all-reduce of "connected") on whether peer mappings work; if any
    rank cannot map its peers (no P2P between these GPUs), every rank uses NCCL instead and a
    warning says so."""

    def __init__(self, group=None, backend=None, fused_reduce_scatter: bool = True):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.be = backend if backend is not None else cuda_ops
        self.fused_rs = fused_reduce_scatter and backend is None and self.world > 1
        self._rs = None
        self._ex = None  # small-value (amax) exchange context
        self._ag = {}    # all-gather contexts by tensor role ("x", "dy")
        self._side = None
        if self.fused_rs:
            self.fused_rs = self._p2p_available()

    def _p2p_available(self) -> bool:
        """Collective: connects the exchange context; True on every rank iff it worked on all."""
        if not torch.cuda.is_available():
            return False
        ex, err = None, None
        try:
            ex = C.TPReduceScatter(self.rank, self.world, 256)
        except C.UFP8Error as e:
            err = e
        handles = [None] * self.world
        dist.all_gather_object(handles, ex.handle if ex is not None else None, group=self.group)
        if ex is not None and all(h is not None for h in handles):
            try:
                ex.connect(handles)
            except C.UFP8Error as e:
                err = e
        ok = torch.tensor([0 if err is not None or ex is None else 1], dtype=torch.int32,
                          device=torch.device("cuda", torch.cuda.current_device()))
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=self.group)
        if int(ok.item()) == 1:
            self._ex = ex
            return True
        if ex is not None:
            ex.close()
        warnings.warn(f"TPGMLP: NVLink peer mappings unavailable ({err or 'on another rank'}); "
                      "using NCCL collectives")
        return False

    def _rs_ctx(self, slot_bytes: int) -> C.TPReduceScatter:
        """Collective: (re)creates the peer-mapped staging when a larger slot is needed."""
        if self._rs is None or self._rs.slot_bytes < slot_bytes:
            if self._rs is not None:
                torch.cuda.synchronize()
                self._rs.close()
            self._rs = self._connect(slot_bytes)
        return self._rs

    def _side_stream(self, device) -> torch.cuda.Stream:
        if self._side is None:
            self._side = torch.cuda.Stream(device=device)
        return self._side

    def copy_reduce_scatter(self, partial: torch.Tensor, between=None):
        """partial [T, d] bf16 (this rank's partial sums): copy engines push block p to rank p on
        the side stream while `between()` (independent work) runs on the current stream, then the
        finish sums; returns (this rank's summed block [T / k, d], between's result)."""
        T, d = partial.shape
        rl = T // self.world
        rs = self._rs_ctx(((rl * d * 2 + 255) // 256) * 256)
        _, epoch = rs.begin()
        main = torch.cuda.current_stream()
        side = self._side_stream(partial.device)
        ready = torch.cuda.Event()
        ready.record(main)
        side.wait_event(ready)
        rs.rs_push_copy(epoch, partial.data_ptr(), partial.stride(0), rl, d, side.cuda_stream)
        partial.record_stream(side)
        done = torch.cuda.Event()
        done.record(side)
        mid = between() if between is not None else None
        main.wait_event(done)
        out = torch.empty((rl, d), dtype=partial.dtype, device=partial.device)
        rs.finish(epoch, rl, d, d, out.data_ptr(), d, main.cuda_stream)
        return out, mid

    def rs_by_copy(self, role: str) -> bool:
        """Whether the reduce-scatter of `role` ("y" or "dx") goes by copy engines (RS_ENGINE)."""
        return RS_ENGINE == "copy" or (RS_ENGINE == "auto" and role == "dx")

    def push_reduce_scatter(self, push, rows: int, cols: int, dtype, device, between=None):
        """Runs `push(slot_table, rank, rows_per_rank)` (a GEMM with the RS_PUSH epilogue over
        all `rows`), then `between()` if given (independent work that runs while the peers'
        pushes land), then the finish; returns (this rank's summed block [rows / k, cols],
        between's result)."""
        rl = rows // self.world
        rs = self._rs_ctx(((rl * cols * 2 + 255) // 256) * 256)
        table, epoch = rs.begin()
        push(table, self.rank, rl)
        mid = between() if between is not None else None
        out = torch.empty((rl, cols), dtype=dtype, device=device)
        rs.finish(epoch, rl, cols, cols, out.data_ptr(), cols, torch.cuda.current_stream().cuda_stream)
        return out, mid

    def close(self) -> None:
        for ctx in (self._rs, self._ex, *self._ag.values()):
            if ctx is not None:
                ctx.close()
        self._rs = self._ex = None
        self._ag = {}

    def _connect(self, slot_bytes: int) -> C.TPReduceScatter:
        """Collective: a new peer-mapped context, its IPC handles exchanged over the group."""
        ctx = C.TPReduceScatter(self.rank, self.world, slot_bytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, ctx.handle, group=self.group)
        ctx.connect(handles)
        ctx.set_copy_lanes(COPY_LANES)
        return ctx

    def gather_tokens_p2p(self, role: str, x: torch.Tensor, fmt: int, amax_t: torch.Tensor):
        """Quantizes this rank's token shard x [T/k, d] straight into its slot of the
        all-gather buffer and starts copying it to every peer on a side stream (AG_ENGINE).
        Returns (the gathered Fp8Tensor [T, d] over the staging memory, the `ag` tuple for
        the consuming GEMM, [the side stream's completion event], the epoch), or None when the
        shapes do not allow it (T/k not a multiple of 256, or T/k * d not of 256 bytes)."""
        rl, d = x.shape
        nbytes = rl * d
        if rl % 256 or nbytes % 256 or self.world > 32:
            return None
        ctx = self._ag.get(role)
        if ctx is None or ctx.slot_bytes != nbytes:  # the gathered view needs slot == block
            if ctx is not None:
                torch.cuda.synchronize()
                ctx.close()
            ctx = self._ag[role] = self._connect(nbytes)
        _, epoch = ctx.begin()
        data, flags = ctx.local(epoch)
        full = _device_bytes(data, (rl * self.world, d), x.device).view(cuda_ops.FP8_DTYPE[fmt])
        q = self.be.quantize(x, fmt, amax_t, out=full[self.rank * rl:(self.rank + 1) * rl])
        main = torch.cuda.current_stream()
        self._side_stream(x.device)
        ready = torch.cuda.Event()
        ready.record(main)
        self._side.wait_event(ready)
        ctx.ag_push(epoch, nbytes, self._side.cuda_stream, AG_ENGINE)
        done = torch.cuda.Event()
        done.record(self._side)
        return cuda_ops.Fp8Tensor(full, q.inv_scale, q.amax), (flags, epoch, self.rank, rl), [done], epoch

    def gathered_still_valid(self, role: str, epoch: int) -> bool:
        """The all-gather buffer of `epoch` is one of two that alternate: it is overwritten by
        the gather two epochs later."""
        ctx = self._ag.get(role)
        return ctx is not None and ctx.epoch - epoch < 2

    def allreduce_max_(self, a: torch.Tensor) -> torch.Tensor:
        """In-place MAX all-reduce of a few amax values (f32, non-negative): over NVLink peer
        memory with the CUDA backend and fused collectives, else a NCCL/gloo all-reduce."""
        if self.fused_rs and a.numel() <= 8:
            if self._ex is None:  # collective: every rank creates it at the same call
                self._ex = self._connect(256)
            a = a.contiguous()
            self._ex.allreduce_max(a.data_ptr(), a.data_ptr(), a.numel(), torch.cuda.current_stream().cuda_stream)
            return a
        dist.all_reduce(a, op=dist.ReduceOp.MAX, group=self.group)
        return a

    def global_amax(self, t: torch.Tensor) -> torch.Tensor:
        return self.allreduce_max_(self.be.amax(t))

    def quant_global(self, t: torch.Tensor, fmt: int):
        return self.be.quantize(t, fmt, self.global_amax(t))

    def quant_global_many(self, tensors_fmts):
        """Quantises several tensors with whole-tensor scales using ONE MAX all-reduce."""
        amaxes = self.allreduce_max_(torch.cat([self.be.amax(t) for t, _ in tensors_fmts]))
        return [self.be.quantize(t, f, amaxes[i:i + 1]) for i, (t, f) in enumerate(tensors_fmts)]

    def all_gather_tokens(self, q):
        """Concatenates every rank's fp8 token shard [T/k, d] into [T, d] (rank order)."""
        local = q.q
        full = torch.empty((local.shape[0] * self.world,) + tuple(local.shape[1:]), dtype=local.dtype,
                           device=local.device)
        dist.all_gather_into_tensor(full.view(torch.uint8), local.contiguous().view(torch.uint8), group=self.group)
        return self.be.Fp8Tensor(full, q.inv_scale, q.amax)

    def reduce_scatter_tokens(self, partial: torch.Tensor) -> torch.Tensor:
        """Sums the ranks' [T, d] partials and leaves rank r its token block [T/k, d]."""
        out = torch.empty((partial.shape[0] // self.world,) + tuple(partial.shape[1:]), dtype=partial.dtype,
                          device=partial.device)
        dist.reduce_scatter_tensor(out, partial.contiguous(), op=dist.ReduceOp.SUM, group=self.group)
        return out


    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        """[rows, ...] on every rank -> [k * rows, ...] in rank order (NCCL / gloo all-gather)."""
        x = x.contiguous()
        full = torch.empty((x.shape[0] * self.world,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(full, x, group=self.group)
        return full

    def reduce_scatter_rows(self, partial: torch.Tensor) -> torch.Tensor:
        """[k * rows, ...] partial sums on every rank -> this rank's summed block [rows, ...]:
        with the NVLink path on 2 ranks the bf16 blocks go by copy engines into the peer's staging
        slot and the finish kernel sums them in fp32 in rank order (copy-engine pushes to several
        peers at once were measured slower than NCCL's); otherwise NCCL / gloo."""
        if self.fused_rs and self.world == 2 and partial.dtype == torch.bfloat16 and partial.is_cuda:
            lead, rest = partial.shape[0], tuple(partial.shape[1:])
            flat = partial.reshape(lead, -1).contiguous()
            if flat.shape[1] % 2 == 0:
                out, _ = self.copy_reduce_scatter(flat)
                return out.reshape((lead // self.world,) + rest)
        return self.reduce_scatter_tokens(partial)


class _GatherRowsFn(torch.autograd.Function):
    """All-gather over the group along dim 0; its gradient is the reduce-scatter."""

    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return tp.all_gather_rows(x)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.reduce_scatter_rows(g.contiguous()), None


class _ScatterRowsFn(torch.autograd.Function):
    """Reduce-scatter over the group along dim 0; its gradient is the all-gather."""

    @staticmethod
    def forward(ctx, partial, tp):
        ctx.tp = tp
        return tp.reduce_scatter_rows(partial)

    @staticmethod
    def backward(ctx, g):
        return ctx.tp.all_gather_rows(g.contiguous()), None


def gather_rows(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """Differentiable all-gather of the ranks' dim-0 blocks (token shards) in rank order."""
    return _GatherRowsFn.apply(x, tp)


def scatter_rows(partial: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """Differentiable reduce-scatter: sums the ranks' partials and keeps this rank's dim-0 block."""
    return _ScatterRowsFn.apply(partial, tp)


class _TPGMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wf, wd, tp: TPContext):
        be = tp.be
        gathered = None
        if tp.fused_rs:
            # one exchange for the three amax values, then x quantized into the all-gather
            # buffer; F1 consumes the peers' blocks as the copy engines deliver them.
            amaxes = tp.allreduce_max_(torch.cat([be.amax(x), be.amax(wf), be.amax(wd)]))
            gathered = tp.gather_tokens_p2p("x", x, C.E4M3, amaxes[0:1])
            qwf = be.quantize(wf, C.E4M3, amaxes[1:2])
            qwd = be.quantize(wd, C.E4M3, amaxes[2:3])
        if gathered is not None:
            qx, ag, done, ctx.x_epoch = gathered
            ug, hid, amax_h = be.gmlp_f1(qx, qwf, ag=ag)
            for ev in done:
                torch.cuda.current_stream().wait_event(ev)
        else:
            if tp.fused_rs:
                qx_local = be.quantize(x, C.E4M3, amaxes[0:1])
            else:
                qx_local, qwf, qwd = tp.quant_global_many([(x, C.E4M3), (wf, C.E4M3), (wd, C.E4M3)])
            qx = tp.all_gather_tokens(qx_local)
            ctx.x_epoch = None
            ug, hid, amax_h = be.gmlp_f1(qx, qwf)
        amax_h = tp.allreduce_max_(amax_h)
        qh = be.quantize(hid, C.E4M3, amax_h)
        if tp.fused_rs and tp.rs_by_copy("y"):
            y, _ = tp.copy_reduce_scatter(be.gmlp_f2(qh, qwd))
        elif tp.fused_rs:
            T, d = qh.q.shape[0], qwd.q.shape[1]
            y, _ = tp.push_reduce_scatter(lambda tab, r, rl: be.gmlp_f2_push(qh, qwd, tab, r, rl), T, d,
                                          torch.bfloat16, qh.q.device)
        else:
            y = tp.reduce_scatter_tokens(be.gmlp_f2(qh, qwd))
        ctx.tp = tp
        ctx.saved = (qx, qwf, ug, qh, qwd)
        return y

    @staticmethod
    def backward(ctx, dy):
        tp = ctx.tp
        be = tp.be
        qx, qwf, ug, qh, qwd = ctx.saved
        ctx.saved = None
        if ctx.x_epoch is not None and not tp.gathered_still_valid("x", ctx.x_epoch):
            raise RuntimeError("TPGMLP: the all-gathered input of this forward pass was overwritten; with "
                               "the NVLink all-gather at most two forward passes may await their backward")
        dyb = dy.to(torch.bfloat16).contiguous()
        gathered = None
        if tp.fused_rs:
            gathered = tp.gather_tokens_p2p("dy", dyb, C.E5M2, tp.global_amax(dyb))
        if gathered is not None:
            qdy, ag, done, _ = gathered
            dug, amax_dug = be.gmlp_b2(qdy, qwd, ug, ag=ag)
            for ev in done:
                torch.cuda.current_stream().wait_event(ev)
        else:
            qdy = tp.all_gather_tokens(tp.quant_global(dyb, C.E5M2))
            dug, amax_dug = be.gmlp_b2(qdy, qwd, ug)
        amax_dug = tp.allreduce_max_(amax_dug)
        dwd = be.gmlp_b1(qh, qdy)
        qdug = be.quantize(dug, C.E5M2, amax_dug)
        if tp.fused_rs and tp.rs_by_copy("dx"):
            dx, dwf = tp.copy_reduce_scatter(be.gmlp_b4(qdug, qwf), between=lambda: be.gmlp_b3(qx, qdug))
        elif tp.fused_rs:
            T, d = qdug.q.shape[1], qwf.q.shape[1]
            dx, dwf = tp.push_reduce_scatter(lambda tab, r, rl: be.gmlp_b4_push(qdug, qwf, tab, r, rl), T, d,
                                             torch.bfloat16, qdug.q.device, between=lambda: be.gmlp_b3(qx, qdug))
        else:
            dx = tp.reduce_scatter_tokens(be.gmlp_b4(qdug, qwf))
            dwf = be.gmlp_b3(qx, qdug)
        return dx, dwf, dwd, None


@config
class TPGMLP(torch.nn.Module):
    """GMLP (ueaj/model/mlp.py:59-115) split over a process group.

    Same constructor as GMLP plus `group` (the tensor-parallel process group; `mesh` is
    accepted as an alias), `device`, and `fused_init` / `down_init` for the two weights.
    Every rank builds the full weights from `rngs` exactly as GMLP does and keeps its slice,
    so a TPGMLP and a GMLP built from the same seed hold the same logical weights.
    `forward` takes this rank's token shard [..., T/k, d] and returns its shard of y.
    """

    def __init__(self, model_d: int, hidden_d: Optional[int] = None, activation_fn: Callable = None,
                 param_dtype: torch.dtype = torch.bfloat16, *, rngs: Rngs, mesh=None, group=None, device=None,
                 fused_init=lecun_normal_init, down_init=zeros_init, backend=None, fused_reduce_scatter: bool = True,
                 full_weights=None):
        """`full_weights` = (wf [2, d, h], wd [h, d]) replaces the construction of the full weights
        from `rngs` (GMLP passes the weights its own projection factories built)."""
        super().__init__()
        hidden_d = 4 * model_d if hidden_d is None else hidden_d
        if group is None and mesh is not None:
            group = tensor_group(mesh) or (mesh if isinstance(mesh, dist.ProcessGroup) else None)
        if hidden_d % dist.get_world_size(group):
            raise ValueError(f"hidden {hidden_d} is not divisible by the tensor-parallel size "
                             f"{dist.get_world_size(group)}")
        self.tp = TPContext(group, backend, fused_reduce_scatter)
        k, r = self.tp.world, self.tp.rank
        if activation_fn is not None:
            from .mlp import swish
            if activation_fn is not swish:
                raise NotImplementedError("the tensor-parallel GMLP fuses swish gating only")
        hl = hidden_d // k
        self.model_d, self.hidden_d, self.hidden_local = model_d, hidden_d, hl
        cpu = torch.device("cpu")
        if full_weights is None:
            full_wf = Einsum("bnd,idh->ibnh", initializer=fused_init, size_dict={"d": model_d, "h": hidden_d, "i": 2},
                             batch_dims="i", rngs=rngs, dtype=param_dtype, sharding=(None, None, "tensor"),
                             device=cpu).w
            full_wd = Einsum("bnh,hd->bnd", initializer=down_init, size_dict={"d": model_d, "h": hidden_d},
                             rngs=rngs, dtype=param_dtype, sharding=("tensor", None), device=cpu).w
        else:
            full_wf, full_wd = full_weights
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else cpu
        # Local shards as Einsum layers over the local hidden width, so optimisers that read
        # Einsum metadata see the shard's canonical layout.
        self.fused_proj = Einsum("bnd,idh->ibnh", initializer=zeros_init, size_dict={"d": model_d, "h": hl, "i": 2},
                                 batch_dims="i", rngs=Rngs(0), dtype=param_dtype, sharding=(None, None, "tensor"),
                                 device=device)
        self.down_proj = Einsum("bnh,hd->bnd", initializer=zeros_init, size_dict={"d": model_d, "h": hl},
                                rngs=Rngs(0), dtype=param_dtype, sharding=("tensor", None), device=device)
        with torch.no_grad():
            self.fused_proj.w.copy_(full_wf[:, :, r * hl:(r + 1) * hl])
            self.down_proj.w.copy_(full_wd[r * hl:(r + 1) * hl, :])

    def shard_tokens(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's contiguous token block of a full [..., d] activation, as [T/k, d]."""
        flat = x.reshape(-1, x.shape[-1])
        n = flat.shape[0]
        if n % self.tp.world:
            raise ValueError(f"{n} tokens are not divisible by the tensor-parallel size {self.tp.world}")
        b = n // self.tp.world
        return flat[self.tp.rank * b:(self.tp.rank + 1) * b].contiguous()

    def forward(self, x_local: torch.Tensor) -> torch.Tensor:
        lead = x_local.shape[:-1]
        x2d = x_local.to(torch.bfloat16).reshape(-1, self.model_d).contiguous()
        wf = self.fused_proj.w if self.fused_proj.w.dtype == torch.bfloat16 else self.fused_proj.w.to(torch.bfloat16)
        wd = self.down_proj.w if self.down_proj.w.dtype == torch.bfloat16 else self.down_proj.w.to(torch.bfloat16)
        return _TPGMLPFn.apply(x2d, wf, wd, self.tp).reshape(*lead, self.model_d)
