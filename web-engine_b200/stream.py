"""Weight streaming from pinned host memory (the loadTransformer analog, src/model/weights.ts:94-131).

    with Streamer(graph, [layer0_bytes, layer1_bytes, ...], slots=2) as st:
        for step in range(steps):
            for l in range(layers):
                w = st.acquire(l)          # device address of layer l, copied on a side stream
                ...ops on graph using w...
                st.release(l)              # the slot can be refilled after that work
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from .graph import Graph


class Streamer:
    def __init__(self, graph: Graph, layers, slots: int = 2, pinned: bool = False):
        """layers: host arrays (numpy, or pinned torch CPU tensors with pinned=True) holding each layer's bytes."""
        self.graph = graph
        self._keep = [np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a for a in layers]
        n = len(self._keep)
        ptrs = (C.c_void_p * n)(*[a.ctypes.data if isinstance(a, np.ndarray) else a.data_ptr() for a in self._keep])
        sizes = (C.c_size_t * n)(*[a.nbytes if isinstance(a, np.ndarray) else a.numel() * a.element_size()
                                   for a in self._keep])
        h = C.c_void_p()
        L.check(graph.ctx, L.lib().we_streamer_create(graph.ctx, ptrs, sizes, n, slots,
                                                      L.STREAM_HOST_PINNED if pinned else 0, C.byref(h)))
        self.h = h

    def acquire(self, layer: int) -> int:
        out = C.c_void_p()
        L.check(self.graph.ctx, L.lib().we_streamer_acquire(self.h, layer, C.byref(out)))
        return out.value

    def release(self, layer: int) -> None:
        L.check(self.graph.ctx, L.lib().we_streamer_release(self.h, layer))

    @property
    def stats(self) -> dict:
        c, b = C.c_uint64(), C.c_uint64()
        L.check(self.graph.ctx, L.lib().we_streamer_stats(self.h, C.byref(c), C.byref(b)))
        return {"copies": c.value, "bytesCopied": b.value}

    def close(self) -> None:
        if self.h:
            L.lib().we_streamer_destroy(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
