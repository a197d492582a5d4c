"""A model of the tensor-parallel P2P protocol (csrc/tp.cu, macrogpt_jax_b200/tp.py), run under
many random interleavings of the ranks' streams: no rank may overwrite a staging slot that a
peer has not finished reading, and every read must see the epoch it waited for.

Each rank has a compute stream and a copy stream (the all-gather pushes).  Ops run atomically
and in stream order; an op whose wait is not yet satisfied blocks its stream.  Memory: per rank
and context, two buffers (epoch parity) of k slots and k arrival flags.  One step (the GMLP
forward + backward of TPGMLP with the default P2P path):

  x all-gather:  compute: quantize x into own slot -> [copy stream: push own slot to every peer,
                 flag each] ; compute: F1 waits for each block's flag and reads it; waits for the
                 copy stream (the event join after F1)
  y reduce-scatter: F2 writes each owner's slot [rank] ; finish: signal, wait all, read own slots
  dY all-gather: as for x ; B2/B1 read the blocks
  dx reduce-scatter: B4 writes ; B3 reads the saved x blocks (forward's buffer) ; finish
"""
import random

import pytest


class Mem:
    def __init__(self, k):
        # [ctx][rank][buffer] -> {"slot": [epoch]*k, "flag": [epoch]*k}
        self.k = k
        self.m = {c: [[{"slot": [0] * k, "flag": [0] * k} for _ in range(2)] for _ in range(k)]
                  for c in ("x", "dy", "rs")}
        self.epoch = {c: [0] * k for c in ("x", "dy", "rs")}


class Violation(AssertionError):
    pass


def _program(r, k, steps, shape="gmlp"):
    """Per-rank op lists: (stream, op, args).  shape "gmlp" is the TPGMLP step; "rs_only" is a
    sequence of back-to-back reduce-scatters (what the C API allows a caller to do)."""
    ops = []
    if shape == "rs_only":
        for _ in range(steps):
            ops.append(("compute", "rs_push", ("y",)))
            ops.append(("compute", "rs_finish", ("y",)))
        return ops
    for _ in range(steps):
        for ctx in ("x", "dy"):
            ops.append(("compute", "begin", (ctx,)))
            ops.append(("compute", "write_own", (ctx,)))
            ops.append(("compute", "record_ready", (ctx,)))
            ops.append(("compute", "gather_read", (ctx,)))      # F1 / B2 (waits per block)
            ops.append(("compute", "join_copy", (ctx,)))
            if ctx == "x":
                ops.append(("compute", "rs_push", ("y",)))        # F2 pushes partial rows
                ops.append(("compute", "rs_finish", ("y",)))      # finish: signal, wait, sum
            else:
                ops.append(("compute", "gather_read_again", ("dy",)))  # B1 reads dY
                ops.append(("compute", "rs_push", ("dx",)))
                ops.append(("compute", "saved_read", ("x",)))     # B3 reads the saved x blocks
                ops.append(("compute", "rs_finish", ("dx",)))
    return ops


def _simulate(k, steps, seed, nbuf=2, mistake=None, shape="gmlp"):
    rng = random.Random(seed)
    mem = Mem(k)
    progs = [_program(r, k, steps, shape) for r in range(k)]
    pc = [0] * k
    # copy-stream queues per rank: pushes appended when the compute stream records "ready"
    copyq = [[] for _ in range(k)]
    state = [{"cur": {}, "pending_push": {}, "rs_epoch": None, "saved_x": []} for _ in range(k)]

    def buf(ctx, owner, e):
        return mem.m[ctx][owner][e % nbuf]

    def try_op(r, op, args):
        st = state[r]
        ctx = args[0]
        if op == "begin":
            mem.epoch[ctx][r] += 1
            st["cur"][ctx] = mem.epoch[ctx][r]
            return True
        e = st["cur"].get(ctx)
        if op == "write_own":
            buf(ctx, r, e)["slot"][r] = e
            return True
        if op == "record_ready":
            for i in range(1, k):
                copyq[r].append((ctx, e, (r - i) % k))
            st["pending_push"][ctx] = e
            return True
        if op == "gather_read" or op == "gather_read_again":
            b = buf(ctx, r, e)
            for s in range(k):
                if s != r and b["flag"][s] != e and mistake != "gather_without_wait":
                    return False
            for s in range(k):
                if b["slot"][s] != e:
                    raise Violation(f"rank {r} reads {ctx} block {s}: epoch {b['slot'][s]} != {e}")
            if ctx == "x":
                st["saved_x"].append(e)
            return True
        if op == "join_copy":
            return not any(c == ctx for c, _, _ in copyq[r])
        if op == "saved_read":
            ex = st["saved_x"].pop(0)
            b = buf("x", r, ex)
            for s in range(k):
                if b["slot"][s] != ex:
                    raise Violation(f"rank {r} reads saved x block {s}: epoch {b['slot'][s]} != {ex}")
            return True
        if op == "rs_push":
            mem.epoch["rs"][r] += 1
            er = mem.epoch["rs"][r]
            st["rs_epoch"] = er
            for o in range(k):
                buf("rs", o, er)["slot"][r] = er  # this rank's partial rows for owner o
            return True
        if op == "rs_finish":
            return _finish(r, st["rs_epoch"])
        raise AssertionError(op)

    def _finish(r, er):
        st = state[r]
        if not st.get("signalled") == er:
            for p in range(k):
                buf("rs", p, er)["flag"][r] = er
            st["signalled"] = er
        b = buf("rs", r, er)
        if any(b["flag"][s] != er for s in range(k)) and mistake != "finish_without_wait":
            return False
        for s in range(k):
            if b["slot"][s] != er:
                raise Violation(f"rank {r} sums rs slot {s}: epoch {b['slot'][s]} != {er}")
        return True

    def try_copy(r):
        ctx, e, p = copyq[r][0]
        b = buf(ctx, p, e)
        b["slot"][r] = e
        b["flag"][r] = e
        copyq[r].pop(0)

    # an op that blocked is retried; a finish that signalled but waits keeps its signal
    while any(pc[r] < len(progs[r]) for r in range(k)) or any(copyq):
        runnable = [("c", r) for r in range(k) if pc[r] < len(progs[r])] + [("q", r) for r in range(k) if copyq[r]]
        rng.shuffle(runnable)
        progressed = False
        for kind, r in runnable:
            if kind == "q":
                try_copy(r)
                progressed = True
                break
            _, op, args = progs[r][pc[r]]
            if try_op(r, op, args):
                pc[r] += 1
                progressed = True
                break
        if not progressed:
            raise Violation("deadlock: every stream waits")


@pytest.mark.parametrize("k", [2, 3, 4, 8])
def test_p2p_protocol_random_interleavings(k):
    for seed in range(60 if k < 8 else 15):
        _simulate(k, steps=4, seed=seed)


@pytest.mark.parametrize("mistake", ["gather_without_wait", "finish_without_wait"])
def test_model_catches_a_missing_wait(mistake):
    """Negative controls: a consumer that does not wait for the arrival flags reads a stale or
    half-written block under some interleaving, and the model reports it."""
    caught = 0
    for seed in range(100):
        try:
            _simulate(3, steps=2, seed=seed, mistake=mistake)
        except Violation:
            caught += 1
    assert caught > 0


def test_single_buffer_is_still_ordered_by_the_step_barriers():
    """Within the TPGMLP step every reuse of a context is separated by a finish and a gathered
    GEMM that wait for all ranks, so even one buffer per context passes every interleaving."""
    for seed in range(60):
        _simulate(3, steps=3, seed=seed, nbuf=1)


def test_back_to_back_reduce_scatters_need_the_second_buffer():
    """A caller may run reduce-scatters back to back with nothing in between: then a fast rank
    that has finished epoch e pushes epoch e+1 while a slow owner still sums epoch e.  With one
    buffer the model catches the overwrite; with the two alternating buffers (the library's
    layout) every interleaving is clean."""
    caught = 0
    for seed in range(200):
        try:
            _simulate(3, steps=4, seed=seed, nbuf=1, shape="rs_only")
        except Violation:
            caught += 1
    assert caught > 0
    for seed in range(200):
        _simulate(3, steps=4, seed=seed, nbuf=2, shape="rs_only")
