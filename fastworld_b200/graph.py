"""CUDA graphs recorded and owned by the engine library.

Contract kept from fastworld/graph.py:13-37: ``capture(fns, warmup, save, load)`` takes
``{key: callable}`` and returns ``{key: graph}`` whose ``replay()`` runs the callable's device
work exactly as an eager call would, and ``state_bytes(tensors)`` sums tensor sizes.

How it works here: a callable issues the engine's launch calls (``fw_chunk``, ``fw_prefill``,
``fw_copy``, op kernels) on torch's current stream.  ``record`` points that stream at a fresh
side stream, opens a thread-local stream capture in the library (``fw_graph_begin``), calls the
callable once and closes the capture (``fw_graph_end``), which instantiates an executable graph
held by the library; ``LibGraph.replay`` launches it on the caller's current stream.  Recording
executes nothing, so it needs no snapshot of the session state; the optional warm-up does run
the callables, and only that phase is bracketed by ``save`` / ``load``.  The engine allocates no
device memory and keeps no lazy state, so there is no memory pool to share between graphs, and
a warm-up is not needed for correctness (``warmup=0`` is valid).

Requirements on a recorded callable: it launches only into buffers that outlive the graph,
allocates nothing on the device and synchronises nothing (the same rules the reference states
for its static runtimes).
"""
from __future__ import annotations

import ctypes
from typing import Callable, Dict, Hashable, Iterable

import torch

from ._lib import check, lib, stream_ptr


class LibGraph:
    """One executable CUDA graph owned by the engine library (``fw_graph``)."""

    __slots__ = ("_g", "_lib", "device")

    def __init__(self, handle: ctypes.c_void_p, device: torch.device):
        self._g, self._lib, self.device = handle, lib(), device

    @classmethod
    def record(cls, fn: Callable[[], object]) -> "LibGraph":
        """Record the device work ``fn`` issues on the current stream (nothing runs)."""
        dev = torch.device("cuda", torch.cuda.current_device())
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        handle = ctypes.c_void_p()
        with torch.cuda.stream(side):
            check(lib().fw_graph_begin(stream_ptr(side)), "fw_graph_begin")
            try:
                fn()
            finally:
                rc = lib().fw_graph_end(stream_ptr(side), ctypes.byref(handle))
        check(rc, "fw_graph_end")
        torch.cuda.current_stream(dev).wait_stream(side)
        return cls(handle, dev)

    def replay(self, stream: torch.cuda.Stream = None) -> None:
        check(self._lib.fw_graph_launch(self._g, stream_ptr(stream)), "fw_graph_launch")

    def num_nodes(self) -> int:
        n = ctypes.c_size_t()
        check(self._lib.fw_graph_nodes(self._g, ctypes.byref(n)), "fw_graph_nodes")
        return n.value

    def __del__(self):
        g, L = getattr(self, "_g", None), getattr(self, "_lib", None)
        if g is not None and g.value and L is not None:
            L.fw_graph_destroy(g)
            self._g = None


def warm_up(fns: Iterable[Callable[[], object]], times: int, save=None, load=None) -> None:
    """Run each callable ``times`` times eagerly, then put the session state back."""
    if times <= 0:
        return
    snapshot = save() if save is not None else None
    for fn in fns:
        for _ in range(times):
            fn()
    if load is not None:
        load(snapshot)


@torch.no_grad()
def capture(fns: Dict[Hashable, Callable[[], object]], warmup: int = 2, save=None,
            load=None) -> Dict[Hashable, LibGraph]:
    """``{key: callable}`` -> ``{key: LibGraph}``; the session state is unchanged on return."""
    warm_up(fns.values(), warmup, save, load)
    graphs = {key: LibGraph.record(fn) for key, fn in fns.items()}
    torch.cuda.synchronize()
    return graphs


def state_bytes(tensors) -> int:
    """Bytes held by the tensors of a session state (non-tensors count zero)."""
    return sum(t.numel() * t.element_size() for t in tensors if isinstance(t, torch.Tensor))
