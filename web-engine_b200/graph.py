"""Graph: device buffers that stay on the GPU, mirroring src/gpu/graph.ts:26-155.

The reference chains WGSL dispatches on one WebGPU queue; here every op of a Graph runs in
order on the CUDA stream of one library context (we_init). Buffers made by ``buffer()`` come
from a pool keyed by size and are zeroed (or overwritten with the given data) on reuse, so
``buffer()`` behaves the same either way (graph.ts:38-54). ``release(mark, keep)`` frees a
step's temporaries, ``free`` one buffer, ``destroy`` everything.
"""
from __future__ import annotations

import ctypes as C
from contextlib import contextmanager
from dataclasses import dataclass

import numpy as np

from . import _lib as L


@dataclass(frozen=True)
class Buffer:
    """A device buffer (GPUBuffer analog): a device address and its size in bytes."""

    ptr: int
    size: int

    @property
    def c(self) -> C.c_void_p:
        return C.c_void_p(self.ptr)


@dataclass(frozen=True)
class Binding:
    """Part of a buffer (graph.ts:24 Binding): offset and size in bytes."""

    buffer: Buffer
    offset: int
    size: int

    @property
    def ptr(self) -> int:
        return self.buffer.ptr + self.offset

    @property
    def c(self) -> C.c_void_p:
        return C.c_void_p(self.ptr)


def addr(b) -> C.c_void_p:
    """Address of a Buffer, Binding, torch tensor, numpy array, raw int pointer, or None."""
    if b is None:
        return C.c_void_p(None)
    if isinstance(b, int):
        return C.c_void_p(b)
    if hasattr(b, "data_ptr"):  # a torch tensor (device, or host for the host-memory entry points)
        return C.c_void_p(b.data_ptr())
    if hasattr(b, "ctypes"):  # a numpy array (host)
        return C.c_void_p(b.ctypes.data)
    return b.c


class Captured:
    """A CUDA graph of a sequence of ops recorded by Graph.capture(): launch() replays it on the graph's stream.
    The buffers the recorded ops created belong to it and keep their addresses until destroy()."""

    def __init__(self, graph: "Graph"):
        self.graph = graph
        self.handle = None

    def launch(self) -> None:
        L.check(self.graph.ctx, L.lib().we_graph_launch(self.graph.ctx, self.handle))

    def destroy(self) -> None:
        if self.handle is not None and self.graph._live:
            L.check(self.graph.ctx, L.lib().we_graph_destroy(self.graph.ctx, self.handle))
        self.handle = None


class Graph:
    def __init__(self, device: int = 0):
        ctx = C.c_void_p()
        rc = L.lib().we_init(device, 0, C.byref(ctx))
        if rc != L.WE_OK:
            raise L.WeError(rc, f"we_init({device}) failed with status {rc} (needs a B200, sm_100)")
        self.ctx = ctx
        self.device = device
        self._live = True

    # ---- buffers ----
    def buffer(self, data) -> Buffer:
        """A device buffer with this data (numpy array / bytes), or zeroed with this many bytes."""
        out = C.c_void_p()
        if isinstance(data, (int, np.integer)):
            L.check(self.ctx, L.lib().we_buffer(self.ctx, int(data), None, C.byref(out)))
            return Buffer(out.value, max(4, (int(data) + 3) // 4 * 4))
        arr = np.ascontiguousarray(data) if not isinstance(data, (bytes, bytearray)) else np.frombuffer(data, np.uint8)
        L.check(self.ctx, L.lib().we_buffer(self.ctx, arr.nbytes, arr.ctypes.data_as(C.c_void_p), C.byref(out)))
        return Buffer(out.value, max(4, (arr.nbytes + 3) // 4 * 4))

    @staticmethod
    def slice(buffer: Buffer, offset: int, size: int) -> Binding:
        """Part of a buffer (offset in bytes; a multiple of 256 like WebGPU's binding rule)."""
        if offset % 256:
            raise ValueError(f"slice offset must be a multiple of 256, got {offset}")
        if offset + size > buffer.size:
            raise ValueError("slice is outside the buffer")
        return Binding(buffer, offset, size)

    def write(self, dst, data) -> None:
        arr = np.ascontiguousarray(data)
        L.check(self.ctx, L.lib().we_write(self.ctx, addr(dst), arr.ctypes.data_as(C.c_void_p), arr.nbytes))

    def copy(self, src, src_offset: int, dst, dst_offset: int, size: int) -> None:
        L.check(self.ctx, L.lib().we_copy(self.ctx, addr(src), src_offset, addr(dst), dst_offset, size))

    def copy_2d(self, src, src_pitch: int, dst, dst_pitch: int, width: int, rows: int) -> None:
        """rows x width bytes from src (rows src_pitch apart) to dst (rows dst_pitch apart), in stream order."""
        L.check(self.ctx, L.lib().we_copy_2d(self.ctx, addr(src), src_pitch, addr(dst), dst_pitch, width, rows))

    def submit(self) -> None:
        """Work is already queued on the stream as it is issued; kept for API parity."""

    def read(self, buffer, nbytes: int | None = None, dtype=np.uint8) -> np.ndarray:
        """Runs everything queued, then copies `nbytes` back (graph.ts:109-119)."""
        n = buffer.size if nbytes is None else nbytes
        out = np.empty(n, dtype=np.uint8)
        L.check(self.ctx, L.lib().we_read(self.ctx, addr(buffer), out.ctypes.data_as(C.c_void_p), n))
        return out.view(dtype)

    def read_into(self, buffer, host_ptr: int, nbytes: int) -> None:
        """Like read(), into caller-owned host memory (e.g. pinned) at `host_ptr`."""
        L.check(self.ctx, L.lib().we_read(self.ctx, addr(buffer), C.c_void_p(host_ptr), nbytes))

    def mark(self) -> int:
        return L.lib().we_mark(self.ctx)

    def release(self, mark: int, keep=()) -> None:
        arr = (C.c_void_p * max(1, len(keep)))(*[b.ptr for b in keep])
        L.check(self.ctx, L.lib().we_release(self.ctx, mark, arr, len(keep)))

    def free(self, buffer: Buffer) -> None:
        L.check(self.ctx, L.lib().we_free(self.ctx, addr(buffer)))

    @property
    def stats(self) -> dict:
        s = L.Stats()
        L.check(self.ctx, L.lib().we_get_stats(self.ctx, C.byref(s)))
        return {"created": s.created, "reused": s.reused, "createdBytes": s.created_bytes, "launches": s.launches,
                "tcGemms": s.tc_gemms, "simtGemms": s.simt_gemms}

    def sync(self) -> None:
        L.check(self.ctx, L.lib().we_sync(self.ctx))

    @contextmanager
    def capture(self):
        """Records the ops issued inside the block as a CUDA graph (we_capture_begin / we_capture_end) instead of
        running them; yields the Captured, which is ready to launch() when the block exits."""
        L.check(self.ctx, L.lib().we_capture_begin(self.ctx))
        cap = Captured(self)
        h = C.c_void_p()
        try:
            yield cap
        except BaseException:
            if L.lib().we_capture_end(self.ctx, C.byref(h)) == L.WE_OK and h.value:
                L.lib().we_graph_destroy(self.ctx, h)
            raise
        L.check(self.ctx, L.lib().we_capture_end(self.ctx, C.byref(h)))
        cap.handle = h

    def set_stream(self, stream: int | None) -> None:
        L.check(self.ctx, L.lib().we_set_stream(self.ctx, C.c_void_p(stream)))

    @property
    def stream(self) -> int:
        return L.lib().we_get_stream(self.ctx) or 0

    @property
    def num_sms(self) -> int:
        return L.lib().we_num_sms(self.ctx)

    def device_error(self) -> int:
        code = C.c_uint32()
        L.check(self.ctx, L.lib().we_device_error(self.ctx, C.byref(code)))
        return code.value

    def destroy(self) -> None:
        if self._live:
            L.lib().we_destroy(self.ctx)
            self._live = False

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.destroy()
