"""The allocation-free linear, we_matmul_fp8_noalloc, against the regular entry point we_matmul.

Callers such as a serving loop whose device memory budget is fixed at start-up, or a host runtime whose
own allocator owns all device memory (a plugin that is handed only streams and pointers), cannot call
cudaMalloc. For them the library keeps the activation split in
one static device array instead of a pooled buffer. This test (the test itself may allocate; the
entry point under test does not) checks that two calls in a row, on different data and sizes, give
the same output as we_matmul on the same inputs, and that a request larger than the static scratch
is refused with a clear message. This file is collected last; it passes alone and after the others.
"""
import ctypes as C

import numpy as np
import pytest

from util import bf16, bf16_round, fast_fp8, randn

pytestmark = pytest.mark.gpu

REL = 1e-5  # the matmul tolerance of the other parity tests


def noalloc(we, graph, xb, m, k, wb, n, csb, yb, y_dtype="bf16", flags=0):
    err = C.create_string_buffer(256)
    rc = we._lib.lib().we_matmul_fp8_noalloc(C.c_void_p(graph.stream), C.c_void_p(xb.ptr), m, k, 0,
                                             C.c_void_p(wb.ptr), n, 1.0, C.c_void_p(csb.ptr), None,
                                             C.c_void_p(yb.ptr), 0, we._lib.DTYPES[y_dtype],
                                             flags | we._lib.NOALLOC_SYNC, err, 256)
    return rc, err.value.decode()


@pytest.mark.parametrize("y_dtype", ["bf16", "f32"])
def test_noalloc_matches_the_pooled_entry_point_on_two_calls(we, y_dtype):
    g = we.Graph(0)
    try:
        ysz = 2 if y_dtype == "bf16" else 4
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
            dt = np.uint16 if y_dtype == "bf16" else np.float32
            a = g.read(y_new, m * n * ysz, dt)
            b = g.read(y_ref, m * n * ysz, dt)
            if y_dtype == "bf16":
                from oracle import oracle as O
                a, b = O.bf16_to_f32(a), O.bf16_to_f32(b)
            rel = float(np.max(np.abs(a.astype(np.float64) - b)) / np.max(np.abs(b)))
            assert rel <= REL, (call, rel)
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
