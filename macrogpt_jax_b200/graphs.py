"""CUDA-graph capture of a whole training step (forward + backward) built from this package's
modules, for workloads small enough that host launch overhead dominates (e.g. GMLP at
d_model 768: six GEMMs of 40-80 us each).

    step = GraphedStep(fn, x, dy)     # warms fn up on a side stream, then captures fn(x, dy)
    out = step(x_new, dy_new)         # copies the inputs into the captured ones, replays

Every kernel of this library is capturable: launches and memsets are stream-ordered, and the
one-time per-device set-up (kernel attributes, occupancy queries, symbol look-ups) happens in
the warm-up, before the capture begins.  The tensor-parallel path is not capturable (it
creates peer-mapped contexts and exchanges IPC handles on first use, and joins side streams).
"""
from __future__ import annotations

from typing import Callable

import torch

from . import ops


class GraphedStep:
    """fn(*inputs) captured once into a CUDA graph on the current device.

    `fn` must be shape-static and must not synchronise with the host.  The captured outputs
    (whatever fn returned during the capture) are overwritten in place by every replay, and
    the inputs passed to __call__ are copied into the static inputs first."""

    def __init__(self, fn: Callable, *example_inputs: torch.Tensor, warmup: int = 3):
        if not example_inputs or not all(t.is_cuda for t in example_inputs):
            raise ValueError("GraphedStep: the example inputs must be CUDA tensors")
        self._static_in = [t.detach().clone() for t in example_inputs]
        saved_timer = ops.get_timer()
        ops.set_timer(None)  # per-launch timing events cannot be recorded inside a capture
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                for _ in range(warmup):
                    fn(*self._static_in)
            torch.cuda.current_stream().wait_stream(side)
            self._graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._graph):
                self._static_out = fn(*self._static_in)
        finally:
            ops.set_timer(saved_timer)

    def __call__(self, *inputs: torch.Tensor):
        if len(inputs) != len(self._static_in):
            raise ValueError(f"GraphedStep: expected {len(self._static_in)} inputs, got {len(inputs)}")
        for dst, src in zip(self._static_in, inputs):
            if src is not dst:
                dst.copy_(src, non_blocking=True)
        self._graph.replay()
        return self._static_out
