"""The library's NCCL communicator (we_comm_* in the C ABI) on one GPU.

- a communicator of one rank: all-gather, reduce-scatter, all-reduce and all-to-all reduce to copies and sums of
  one operand, checked bit for bit; the host-blob all-gather and max-over-ranks helpers;
- failure detection without a GPU fault: a communicator of two ranks whose second rank never joins. Init must give
  up within its host deadline with WE_ETIMEOUT (the communicator is aborted), and the context stays usable. No
  kernel of the failed communicator ever runs; the failure is made on the host (a rank that never joins).
"""
import os
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_single_rank_collectives(we, graph):
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    comm = we.comm.Comm(graph, 0, 1, we.comm.unique_id(), timeout_ms=30000)
    try:
        x = np.random.default_rng(0).standard_normal(4096).astype(np.float32)
        xb = graph.buffer(x)
        y = graph.buffer(x.nbytes)
        comm.all_gather(xb, y, x.nbytes)
        assert np.array_equal(graph.read(y, x.nbytes, np.float32), x)
        comm.reduce_scatter(xb, y, x.size, "f32")
        assert np.array_equal(graph.read(y, x.nbytes, np.float32), x)
        comm.all_reduce(xb, y, x.size, "f32", "max")
        assert np.array_equal(graph.read(y, x.nbytes, np.float32), x)
        comm.all_to_all(xb, y, x.nbytes)
        assert np.array_equal(graph.read(y, x.nbytes, np.float32), x)
        assert comm.all_gather_bytes(b"0123456789abcdef") == [b"0123456789abcdef"]
        assert comm.max_over_ranks(2.5) == 2.5
        comm.barrier()
    finally:
        comm.destroy()
    assert graph.device_error() == 0


def _never_joins(q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    from conftest import load_package

    we = load_package()
    g = we.Graph(0)
    t0 = time.monotonic()
    try:
        we.comm.Comm(g, 0, 2, we.comm.unique_id(), timeout_ms=3000)
        q.put(("joined", 0, time.monotonic() - t0, 0))
    except we.comm.CommError as exc:
        elapsed = time.monotonic() - t0
        b = g.buffer(np.arange(16, dtype=np.float32))  # the context is still usable
        ok = np.array_equal(g.read(b, 64, np.float32), np.arange(16, dtype=np.float32)) and g.device_error() == 0
        q.put(("error", exc.code, elapsed, int(ok)))
    g.destroy()


def test_a_rank_that_never_joins_times_out(we):
    """Rank 1 of two never calls we_comm_init: rank 0's init gives up after its 3 s deadline with WE_ETIMEOUT. The
    rank runs in a child process that the test can end if NCCL's abort itself were to block (host side only)."""
    import multiprocessing

    mp = multiprocessing.get_context("spawn")
    q = mp.SimpleQueue()
    p = mp.Process(target=_never_joins, args=(q,))
    p.start()
    p.join(timeout=90)
    if p.is_alive():
        p.kill()
        p.join()
        pytest.fail("the rank did not return from a communicator init whose peer never joined")
    kind, code, elapsed, ok = q.get()
    assert kind == "error" and code == we._lib.WE_ETIMEOUT, (kind, code)
    assert elapsed < 30 and ok, (elapsed, ok)
