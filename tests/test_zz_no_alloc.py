"""The allocation-free linear, we_matmul_fp8_noalloc, against the regular entry point we_matmul and the oracle.

Callers such as a serving loop whose device memory budget is fixed at start-up, or a host runtime whose
own allocator owns all device memory (a plugin that is handed only streams and pointers), cannot call
cudaMalloc. For them the library keeps the activation split in one static device array instead of a pooled
buffer. These tests (the tests themselves may allocate; the entry point under test does not) check that:
- two calls in a row, on different data and sizes, give the same output as we_matmul on the same inputs;
- one case matches the float64 oracle within the matmul tolerance of the other parity tests;
- a warmed-up call leaves the device's free memory unchanged (it allocates nothing);
- a call without WE_NOALLOC_SYNC returns before the work is done and gives the same output once the stream is
  synchronised;
- a request larger than the static scratch is refused with a clear message.
This file is collected last; it passes alone and after the others.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, fast_fp8, randn

pytestmark = pytest.mark.gpu

REL = 1e-5  # the matmul tolerance of the other parity tests


def noalloc(we, graph, xb, m, k, wb, n, csb, yb, y_dtype="bf16", flags=None):
    err = C.create_string_buffer(256)
    flags = we._lib.NOALLOC_SYNC if flags is None else flags
    rc = we._lib.lib().we_matmul_fp8_noalloc(C.c_void_p(graph.stream), C.c_void_p(xb.ptr), m, k, 0,
                                             C.c_void_p(wb.ptr), n, 1.0, C.c_void_p(csb.ptr), None,
                                             C.c_void_p(yb.ptr), 0, we._lib.DTYPES[y_dtype], flags, err, 256)
    return rc, err.value.decode()


def as_f32(a, y_dtype):
    return O.bf16_to_f32(a) if y_dtype == "bf16" else a


@pytest.mark.parametrize("y_dtype", ["bf16", "f32"])
def test_noalloc_matches_the_pooled_entry_point_on_two_calls(we, y_dtype):
    g = we.Graph(0)
    try:
        ysz = 2 if y_dtype == "bf16" else 4
        dt = np.uint16 if y_dtype == "bf16" else np.float32
        for call, (m, n, k, seed) in enumerate([(300, 520, 768, 1), (2304, 1024, 3072, 2)]):
            x = bf16_round(randn(m * k, seed))
            w = fast_fp8(n * k, seed + 10)
            cs = (np.abs(randn(n, seed + 20, 0.01)) + np.float32(1e-3)).astype(np.float32)
            xb, wb, csb = g.buffer(bf16(x)), g.buffer(w), g.buffer(cs)
            y_ref, y_new = g.buffer(m * n * ysz), g.buffer(m * n * ysz)
            we.kernels.matmul(g, xb, wb, y_ref, m, n, k, 1.0, x_dtype="bf16", w_dtype="fp8", y_dtype=y_dtype,
                              chan_scale=csb)
            rc, msg = noalloc(we, g, xb, m, k, wb, n, csb, y_new, y_dtype)
            assert rc == we._lib.WE_OK, msg
            a = as_f32(g.read(y_new, m * n * ysz, dt), y_dtype)
            b = as_f32(g.read(y_ref, m * n * ysz, dt), y_dtype)
            rel = float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b)))
            assert rel <= REL, (call, rel)
            if call == 0 and y_dtype == "f32":  # the float64 oracle on the same bf16 inputs
                want = O.matmul(x, O.FP8, w, m, n, k, chan_scale=cs)
                assert O.rel_error(a, want) < REL
    finally:
        g.destroy()


def test_noalloc_allocates_nothing_and_runs_asynchronously(we):
    torch = pytest.importorskip("torch")
    g = we.Graph(0)
    try:
        m, n, k = 1024, 768, 1536
        x = bf16_round(randn(m * k, 5))
        w = fast_fp8(n * k, 6)
        cs = (np.abs(randn(n, 7, 0.01)) + np.float32(1e-3)).astype(np.float32)
        xb, wb, csb = g.buffer(bf16(x)), g.buffer(w), g.buffer(cs)
        y_ref, y_new = g.buffer(m * n * 4), g.buffer(m * n * 4)
        we.kernels.matmul(g, xb, wb, y_ref, m, n, k, 1.0, x_dtype="bf16", w_dtype="fp8", y_dtype="f32",
                          chan_scale=csb)
        # warm-up: the first call in this context may load the library's module (and its static array)
        rc, msg = noalloc(we, g, xb, m, k, wb, n, csb, y_new, "f32")
        assert rc == we._lib.WE_OK, msg
        g.sync()
        free0, _ = torch.cuda.mem_get_info(0)
        for _ in range(3):  # queued without waiting: WE_NOALLOC_SYNC not given
            rc, msg = noalloc(we, g, xb, m, k, wb, n, csb, y_new, "f32", flags=0)
            assert rc == we._lib.WE_OK, msg
        g.sync()
        free1, _ = torch.cuda.mem_get_info(0)
        assert free1 == free0, (free0, free1)
        a = g.read(y_new, m * n * 4, np.float32)
        b = g.read(y_ref, m * n * 4, np.float32)
        assert float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b))) <= REL
        assert g.device_error() == 0
    finally:
        g.destroy()


def test_noalloc_refuses_more_than_its_static_scratch(we):
    g = we.Graph(0)
    try:
        k = 3072
        m = we._lib.NOALLOC_SCRATCH_BYTES // (2 * k) + 1  # two e4m3 planes of m x k no longer fit
        xb, wb, csb, yb = g.buffer(16), g.buffer(k * 16), g.buffer(64), g.buffer(16)
        rc, msg = noalloc(we, g, xb, m, k, wb, 16, csb, yb)
        assert rc == we._lib.WE_EINVAL
        assert "static scratch" in msg and str(we._lib.NOALLOC_SCRATCH_BYTES) in msg
    finally:
        g.destroy()
