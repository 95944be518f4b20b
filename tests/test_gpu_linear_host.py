"""GPU tests of the host-memory linear (we_linear_host): the upload, the linear of src/model/ops.ts:61-73 and the
read-back of src/gpu/graph.ts:108-119 in one call, with row chunks whose copies overlap the GEMMs."""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, make_linear, randn

pytestmark = pytest.mark.gpu


def _host_bf16(torch, values, pinned=True):
    t = torch.from_numpy(bf16(values).view(np.int16).copy())
    return t.pin_memory() if pinned else t


def _bits(t):
    return t.numpy().view(np.uint16)


def _device_linear(we, graph, x_bits, lin, m, y_dtype="bf16"):
    """The same linear on the device path: upload, we_linear_forward, read."""
    mark = graph.mark()
    y = we.linear(graph, graph.buffer(x_bits), lin, m, x_dtype="bf16", y_dtype=y_dtype)
    got = graph.read(y, m * lin.n * (2 if y_dtype == "bf16" else 4), np.uint16 if y_dtype == "bf16" else np.float32)
    graph.release(mark)
    return got


@pytest.mark.parametrize("chunk_rows", [0, 256, 300, 1000, 4096])
def test_linear_host_equals_the_device_linear(we, graph, chunk_rows):
    """Ragged m over chunks of 128 (default for m = 1000), 256, 300 (not a tile multiple), m and more than m:
    every row of y is the bf16 linear of its x row, bit for bit as the device path computes it."""
    import torch

    m, n, k = 1000, 1536, 3072
    _, lin = make_linear(we, graph, n, k, 11)
    x = bf16_round(randn(m * k, 12))
    xh = _host_bf16(torch, x)
    yh = torch.zeros(m * n, dtype=torch.int16).pin_memory()
    we.linear_host(graph, xh, lin, m, yh, chunk_rows=chunk_rows)
    want = _device_linear(we, graph, bf16(x), lin, m)
    assert np.array_equal(_bits(yh), want)


def test_linear_host_matches_the_oracle(we, graph):
    """Small case against the float64 oracle: y = x . (q * chan_scale)^T, rounded once to bf16."""
    import torch

    m, n, k = 200, 256, 512
    host, lin = make_linear(we, graph, n, k, 21)
    x = bf16_round(randn(m * k, 22))
    xh = _host_bf16(torch, x)
    yh = torch.zeros(m * n, dtype=torch.float32).pin_memory()
    we.linear_host(graph, xh, lin, m, yh, y_dtype="f32", chunk_rows=128)
    want = O.matmul(x, O.FP8, host["bytes"], m, n, k, chan_scale=host["chan_scale"])
    assert O.rel_error(yh.numpy(), want) < 1e-5


def test_linear_host_with_pageable_buffers(we, graph):
    """numpy (pageable) host arrays: the copies do not overlap, the result is the same."""
    m, n, k = 384, 512, 1024
    _, lin = make_linear(we, graph, n, k, 31)
    x = bf16(bf16_round(randn(m * k, 32)))
    y = np.zeros(m * n, np.uint16)
    we.linear_host(graph, x, lin, m, y, chunk_rows=128)
    assert np.array_equal(y, _device_linear(we, graph, x, lin, m))


def test_linear_host_with_lora(we, graph):
    """A LoRA linear through the chunks: each chunk is we_linear_forward of its rows (the narrow down projection
    may split over K differently for fewer rows), so the result matches within f32 rounding."""
    import torch

    m, n, k, rank = 512, 256, 4096, 16
    _, lin0 = make_linear(we, graph, n, k, 41)
    down = bf16(bf16_round(randn(rank * k, 42, 0.05)))
    up = bf16(bf16_round(randn(n * rank, 43, 0.05)))
    lin = we.Linear(lin0.buffer, "fp8", 1.0, n, k, chan_scale=lin0.chan_scale,
                    lora=(we.Linear(graph.buffer(down), "bf16", 1.0, rank, k),
                          we.Linear(graph.buffer(up), "bf16", 0.5, n, rank)))
    x = bf16_round(randn(m * k, 44))
    xh = _host_bf16(torch, x)
    yh = torch.zeros(m * n, dtype=torch.float32).pin_memory()
    we.linear_host(graph, xh, lin, m, yh, y_dtype="f32", chunk_rows=128)
    want = _device_linear(we, graph, bf16(x), lin, m, y_dtype="f32")
    assert O.rel_error(yh.numpy(), want.astype(np.float64)) < 1e-6


def test_linear_host_edges(we, graph):
    """m = 0 does nothing; a bad LoRA shape is refused before anything is copied; no host round trip while
    capturing a graph."""
    import torch

    n, k = 256, 512
    _, lin = make_linear(we, graph, n, k, 51)
    we.linear_host(graph, None, lin, 0, None)
    wb = graph.buffer(n * k)
    bad = we.Linear(wb, "fp8", 1.0, n, k, lora=(we.Linear(wb, "bf16", 1.0, 6, k), we.Linear(wb, "bf16", 1.0, n, 6)))
    xh = torch.zeros(128 * k, dtype=torch.int16).pin_memory()
    yh = torch.zeros(128 * n, dtype=torch.int16).pin_memory()
    with pytest.raises(we._lib.WeError, match="LoRA shapes do not fit the linear layer"):
        we.linear_host(graph, xh, bad, 128, yh)
    g = we.Graph(0)
    try:
        _, lin_g = make_linear(we, g, n, k, 52)
        with pytest.raises(we._lib.WeError, match="while capturing"):
            with g.capture():
                we.linear_host(g, xh, lin_g, 128, yh)
        we.linear_host(g, xh, lin_g, 128, yh)  # the context works again after the failed capture
    finally:
        g.destroy()
