"""One-GPU tests of the peer-memory exchange (we_peer_*): its copy rule on a group of one rank, and its bounded
barrier. A group of two whose second rank never runs (both members map to this rank's own memory) makes the
barrier wait for a flag that nothing sets: the kernel must give up after its timeout, record
DEV_ERR_TIMEOUT_PEER (5) in the context's error word and leave the context usable. The two-GPU exchange is
covered by test_gpu_sequence.py."""
import ctypes as C
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

DEV_ERR_TIMEOUT_PEER = 5


def _group(we, g, rank, world, nbytes, blobs_of=None):
    L = we._lib
    h = C.c_void_p()
    L.check(g.ctx, L.lib().we_peer_create(g.ctx, rank, world, nbytes, C.byref(h)))
    blob = (C.c_ubyte * L.PEER_HANDLE_BYTES)()
    L.check(g.ctx, L.lib().we_peer_export(h, blob))
    allb = (C.c_ubyte * (L.PEER_HANDLE_BYTES * world)).from_buffer_copy(bytes(blob) * world)
    L.check(g.ctx, L.lib().we_peer_open(h, allb))
    return h


def _exchange(we, g, h, copies, timeout_ns=0):
    L = we._lib
    arr = (L.PeerCopy * len(copies))(*[L.PeerCopy(**c) for c in copies])
    L.check(g.ctx, L.lib().we_peer_exchange(g.ctx, h, arr, len(copies), timeout_ns))


def test_exchange_on_one_rank_is_the_copy_rule(we):
    """world 1: the head scatter lays q out as [t, heads, bytes] (all heads are this rank's), the gather of that
    block brings the same rows back, the row all-gather copies the rows; bit for bit."""
    seq = we.sequence
    g = we.Graph(0)
    h = None
    try:
        t, heads, hb = 37, 3, 256
        rng = np.random.default_rng(3)
        q = rng.integers(0, 256, t * heads * hb, dtype=np.uint8)
        qb = g.buffer(q)
        size = 3 * q.size
        h = _group(we, g, 0, 1, size)
        region = we._lib.lib().we_peer_region(h)
        _exchange(we, g, h, [seq.scatter_copy(qb.ptr, t, heads, hb, 1, 0)])
        _exchange(we, g, h, [seq.gather_copy(region, t, heads, hb, 1, q.size)])
        _exchange(we, g, h, [seq.rows_copy(qb.ptr, q.size, 2 * q.size)])
        got = g.read(region, size, np.uint8)
        assert np.array_equal(got[:q.size], q) and np.array_equal(got[q.size:2 * q.size], q)
        assert np.array_equal(got[2 * q.size:], q)
        assert g.device_error() == 0
    finally:
        if h is not None:
            we._lib.lib().we_peer_destroy(h)
        g.destroy()


def test_exchange_refuses_bad_copies(we):
    seq = we.sequence
    g = we.Graph(0)
    h = None
    try:
        h = _group(we, g, 0, 1, 4096)
        src = g.buffer(np.zeros(8192, np.uint8))
        with pytest.raises(we._lib.WeError, match="past the exchange region"):
            _exchange(we, g, h, [seq.rows_copy(src.ptr, 8192)])
        bad = seq.rows_copy(src.ptr, 1024)
        bad["chunk_bytes"] = 24
        with pytest.raises(we._lib.WeError, match="16-byte"):
            _exchange(we, g, h, [bad])
        with pytest.raises(we._lib.WeError, match="1 to 8 ranks"):
            _group(we, g, 0, 9, 4096)
    finally:
        if h is not None:
            we._lib.lib().we_peer_destroy(h)
        g.destroy()


def test_barrier_gives_up_when_a_rank_never_comes(we):
    seq = we.sequence
    g = we.Graph(0)
    h = None
    try:
        h = _group(we, g, 0, 2, 8192)  # rank 1 maps to this rank's memory and never runs its half
        src = g.buffer(np.arange(1024, dtype=np.uint8) % 251)
        t0 = time.perf_counter()
        _exchange(we, g, h, [seq.rows_copy(src.ptr, 1024)], timeout_ns=50_000_000)  # 50 ms
        code = g.device_error()  # waits for the kernel
        elapsed = time.perf_counter() - t0
        assert code == DEV_ERR_TIMEOUT_PEER, code
        assert 0.04 < elapsed < 10.0, elapsed
        # the context still runs work after the timeout
        b = g.buffer(np.arange(4, dtype=np.float32))
        assert g.read(b, 16, np.float32).tolist() == [0, 1, 2, 3]
        assert g.device_error() == 0
    finally:
        if h is not None:
            we._lib.lib().we_peer_destroy(h)
        g.destroy()
