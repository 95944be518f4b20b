"""Collectives for the multi-GPU paths, through the library's C ABI (we_comm_*, NCCL over NVLink / NVSwitch).

One process per GPU, one communicator per library context. Rank 0 makes the unique id; `rendezvous` carries it to
the other ranks over a plain TCP connection (any other host channel works as well: the id is 128 bytes). Every
collective is queued on the context's stream and works on device buffers (graph Buffers, raw device addresses, or
anything `graph.addr` accepts). A host deadline bounds every call: a rank that never joins or an NCCL failure
aborts the communicator and raises CommError with WE_ETIMEOUT / WE_ENCCL, instead of hanging the caller.
"""
from __future__ import annotations

import ctypes as C
import importlib.util
import os
import socket
import struct
import time

import numpy as np

from . import _lib as L
from .graph import Graph, addr


class CommError(L.WeError):
    """A collective failed or timed out; the communicator is aborted."""


def _prefer_wheel_nccl() -> None:
    """Points the library at the NCCL of the NVIDIA wheel (nvidia-nccl-cu12) when one is installed and the caller
    chose none (WE_NCCL_LIBRARY): a process holds a single libnccl.so.2, and other libraries loaded into it later
    (a framework built against that wheel) need the wheel's version, which can be newer than the system's."""
    if os.environ.get("WE_NCCL_LIBRARY"):
        return
    try:
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        return
    for base in (spec.submodule_search_locations or []) if spec else []:
        path = os.path.join(base, "lib", "libnccl.so.2")
        if os.path.exists(path):
            os.environ["WE_NCCL_LIBRARY"] = path
            return


def unique_id() -> bytes:
    """A fresh NCCL unique id (rank 0 makes it once per communicator)."""
    _prefer_wheel_nccl()
    buf = (C.c_ubyte * L.COMM_ID_BYTES)()
    rc = L.lib().we_comm_unique_id(buf)
    if rc != L.WE_OK:
        raise CommError(rc, "we_comm_unique_id failed (is NCCL installed?)")
    return bytes(buf)


def _recv_exact(sock: socket.socket, n: int) -> bytes:
    out = b""
    while len(out) < n:
        chunk = sock.recv(n - len(out))
        if not chunk:
            raise ConnectionError("the rendezvous peer closed the connection")
        out += chunk
    return out


def rendezvous(rank: int, world: int, host: str, port: int, payload: bytes | None = None,
               timeout_s: float = 60.0) -> bytes:
    """Rank 0 listens on (host, port) and sends `payload` (default: a new unique id) to the other world - 1 ranks,
    which connect (retrying until timeout_s) and return it. Returns the payload on every rank."""
    deadline = time.monotonic() + timeout_s
    if rank == 0:
        data = payload if payload is not None else unique_id()
        with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as srv:
            srv.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            srv.bind((host, port))
            srv.listen(world)
            for _ in range(world - 1):
                srv.settimeout(max(0.1, deadline - time.monotonic()))
                conn, _ = srv.accept()
                with conn:
                    conn.sendall(struct.pack("<I", len(data)) + data)
        return data
    while True:
        try:
            with socket.create_connection((host, port), timeout=max(0.1, deadline - time.monotonic())) as s:
                n = struct.unpack("<I", _recv_exact(s, 4))[0]
                return _recv_exact(s, n)
        except OSError:
            if time.monotonic() > deadline:
                raise
            time.sleep(0.05)


class Comm:
    """A communicator of `world` ranks on this graph's device and stream."""

    def __init__(self, graph: Graph, rank: int, world: int, uid: bytes, timeout_ms: int = 60000):
        if len(uid) != L.COMM_ID_BYTES:
            raise ValueError(f"the unique id has {L.COMM_ID_BYTES} bytes")
        self.graph, self.rank, self.world = graph, rank, world
        _prefer_wheel_nccl()
        h = C.c_void_p()
        idb = (C.c_ubyte * L.COMM_ID_BYTES).from_buffer_copy(uid)
        rc = L.lib().we_comm_init(graph.ctx, world, rank, idb, timeout_ms, C.byref(h))
        if rc != L.WE_OK:
            msg = L.lib().we_last_error(graph.ctx)
            raise CommError(rc, (msg.decode() if msg else "") or f"we_comm_init failed ({rc})")
        self.handle = h

    def _check(self, rc: int) -> None:
        if rc != L.WE_OK:
            msg = L.lib().we_comm_last_error(self.handle)
            raise CommError(rc, (msg.decode() if msg else "") or f"collective failed ({rc})")

    def all_gather(self, src, dst, nbytes: int) -> None:
        """dst [world * nbytes] = every rank's src [nbytes] in rank order."""
        self._check(L.lib().we_all_gather(self.handle, addr(src), addr(dst), nbytes))

    def reduce_scatter(self, src, dst, count: int, dtype: str = "f32") -> None:
        """dst [count] = this rank's slice of the sum over ranks of src [world * count]."""
        self._check(L.lib().we_reduce_scatter(self.handle, addr(src), addr(dst), count, L.DTYPES[dtype]))

    def all_reduce(self, src, dst, count: int, dtype: str = "f32", op: str = "sum") -> None:
        self._check(L.lib().we_all_reduce(self.handle, addr(src), addr(dst), count, L.DTYPES[dtype],
                                          L.REDUCE_MAX if op == "max" else L.REDUCE_SUM))

    def all_to_all(self, src, dst, bytes_per_rank: int) -> None:
        """Chunk p of dst = chunk `rank` of rank p's src (equal chunks of bytes_per_rank)."""
        self._check(L.lib().we_all_to_all(self.handle, addr(src), addr(dst), bytes_per_rank))

    def barrier(self) -> None:
        self._check(L.lib().we_comm_barrier(self.handle))

    def wait(self) -> None:
        self._check(L.lib().we_comm_wait(self.handle))

    def all_gather_bytes(self, blob: bytes) -> list[bytes]:
        """Every rank's host blob (all the same length), in rank order, through device memory."""
        n = len(blob)
        src = self.graph.buffer(np.frombuffer(blob, np.uint8))
        dst = self.graph.buffer(self.world * max(n, 4))
        self.all_gather(src, dst, n)
        out = self.graph.read(dst, self.world * n).tobytes()
        self.graph.free(src)
        self.graph.free(dst)
        return [out[i * n:(i + 1) * n] for i in range(self.world)]

    def max_over_ranks(self, value: float) -> float:
        """The largest host value over the ranks (timings are reported as the max over ranks)."""
        if self.world == 1:
            return float(value)
        b = self.graph.buffer(np.array([value], np.float32))
        self.all_reduce(b, b, 1, "f32", "max")
        v = float(self.graph.read(b, 4, np.float32)[0])
        self.graph.free(b)
        return v

    def abort(self) -> None:
        if self.handle is not None:
            L.lib().we_comm_abort(self.handle)

    def destroy(self) -> None:
        if self.handle is not None:
            L.lib().we_comm_destroy(self.handle)
            self.handle = None
