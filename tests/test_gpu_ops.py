"""GPU tests of the Graph substrate and the operator API (src/gpu/graph.ts, src/model/ops.ts), mirroring
tests/gpu/graph.test.ts and tests/gpu/lora.test.ts, plus the q/k path of a block (src/model/block.ts:53-56)."""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, fast_fp8, lcg_floats, randn

pytestmark = pytest.mark.gpu


# ---------------- Graph: tests/gpu/graph.test.ts ----------------
def test_slice_binds_part_of_a_buffer(we, graph):  # graph.test.ts:7-16
    data = graph.buffer(np.arange(192, dtype=np.float32))
    s1, s2 = we.Graph.slice(data, 256, 256), we.Graph.slice(data, 512, 256)
    out = graph.buffer(64 * 4)
    graph.copy(s1, 0, out, 0, 256)
    got = graph.read(out, 256, np.float32)
    assert got[0] == 64 and got[63] == 127
    got2 = graph.read(s2, 256, np.float32)
    assert got2[0] == 128 and got2[63] == 191
    with pytest.raises(ValueError):
        we.Graph.slice(data, 100, 4)


def test_copy_in_order(we, graph):  # graph.test.ts:18-24
    a = graph.buffer(np.array([1, 2, 3, 4], np.float32))
    b = graph.buffer(8 * 4)
    graph.copy(a, 0, b, 16, 16)
    assert graph.read(b, 32, np.float32).tolist() == [0, 0, 0, 0, 1, 2, 3, 4]


def test_release_keeps_what_is_asked_for(we):  # graph.test.ts:26-36
    g = we.Graph(0)
    try:
        before = g.buffer(4)
        mark = g.mark()
        g.buffer(4)
        kept = g.buffer(np.array([7], np.float32))
        g.release(mark, [kept])
        assert g.mark() == mark + 1
        assert g.read(kept, 4, np.float32)[0] == 7
        g.free(before)
    finally:
        g.destroy()


def test_reuses_released_buffers_of_the_same_size(we):  # graph.test.ts:38-48
    g = we.Graph(0)
    try:
        mark = g.mark()
        first = g.buffer(4096)
        g.release(mark)
        again = g.buffer(4096)
        assert again.ptr == first.ptr
        s = g.stats
        assert s["created"] == 1 and s["reused"] == 1
        assert g.buffer(8192).ptr != first.ptr
    finally:
        g.destroy()


def test_zeroes_or_refills_a_reused_buffer(we):  # graph.test.ts:50-62
    g = we.Graph(0)
    try:
        mark = g.mark()
        g.buffer(np.arange(1, 1001, dtype=np.float32))
        g.release(mark)
        z = g.buffer(4000)
        assert np.all(g.read(z, 4000, np.float32) == 0)
        mark = g.mark()
        g.buffer(np.arange(1, 1001, dtype=np.float32))
        g.release(mark)
        f = g.buffer(np.full(1000, 5, np.float32))
        assert np.all(g.read(f, 4000, np.float32) == 5)
    finally:
        g.destroy()


# ---------------- linear / LoRA: src/model/ops.ts:61-73, tests/gpu/lora.test.ts ----------------
def test_linear_with_bias_f32(we, graph):
    m, n, k = 33, 96, 128
    x = lcg_floats(m * k, 1)
    w = fast_fp8(n * k, 2)
    bias = randn(n, 3)
    xb, wb, bb = graph.buffer(x), graph.buffer(w), graph.buffer(bias)
    y = we.linear(graph, xb, we.Linear(wb, "fp8", 0.01, n, k, bias=bb), m)
    got = graph.read(y, m * n * 4, np.float32)
    want = O.matmul(x, O.FP8, w, m, n, k, scale=0.01).reshape(m, n) + bias
    assert O.rel_error(got, want) < 1e-5


@pytest.mark.parametrize("x_dtype", ["f32", "bf16"])
def test_linear_with_lora(we, graph, x_dtype):
    """y = x W^T + up.scale (x down^T) up^T; the down projection is narrow with a long K, so
    narrowLinear splits it over K (ops.ts:48-58)."""
    m, n, k, rank = 40, 256, 4096, 16
    x = bf16_round(lcg_floats(m * k, 4))
    w = fast_fp8(n * k, 5)
    down = bf16_round(randn(rank * k, 6, 0.05))
    up = bf16_round(randn(n * rank, 7, 0.05))
    assert we.k_split_for(m, rank, k) > 1
    xb = graph.buffer(x if x_dtype == "f32" else bf16(x))
    lin = we.Linear(graph.buffer(w), "fp8", 0.002, n, k,
                    lora=(we.Linear(graph.buffer(bf16(down)), "bf16", 1.0, rank, k),
                          we.Linear(graph.buffer(bf16(up)), "bf16", 0.75, n, rank)))
    before = graph.stats["launches"]
    y = we.linear(graph, xb, lin, m, x_dtype=x_dtype)
    assert graph.stats["launches"] - before >= 3
    got = graph.read(y, m * n * 4, np.float32)
    base = O.matmul(x, O.FP8, w, m, n, k, scale=0.002)
    t = O.matmul(x, O.BF16, bf16(down), m, rank, k)
    delta = O.matmul(t.astype(np.float32), O.BF16, bf16(up), m, n, rank, scale=0.75)
    assert O.rel_error(got, base + delta) < 1e-5


def test_linear_refuses_lora_that_does_not_fit(we, graph):  # ops.ts:68
    n, k = 64, 128
    wb = graph.buffer(n * k)
    bad = we.Linear(wb, "fp8", 1.0, n, k, lora=(we.Linear(wb, "bf16", 1.0, 6, k), we.Linear(wb, "bf16", 1.0, n, 6)))
    with pytest.raises(we._lib.WeError, match="LoRA shapes do not fit the linear layer"):
        we.linear(graph, graph.buffer(4 * k * 4), bad, 4)


# ---------------- norm / rotate ops and the block's q/k path ----------------
def test_norm_and_no_mod(we, graph):
    rows, d = 64, 3072
    x = randn(rows * d, 1)
    w = randn(d, 2, 0.1)
    out = we.norm(graph, graph.buffer(x), graph.buffer(w), rows, d, we.no_mod(graph, d))
    got = graph.read(out, rows * d * 4, np.float32)
    assert np.max(np.abs(got - O.rmsnorm(x, w, None, None, 1e-5, 1.0))) < 1e-5


def test_block_qk_path_linear_norm_rotate(we, graph):
    """attend()'s projected(): q = rotate(norm(linear(h, wq), qNorm, rows*heads, 128)) with bf16
    activations and the config-3 RoPE (axes 16/56/56, theta 1e4), unfused ops vs the fused kernel."""
    text, side, heads, hidden = 8, 8, 4, 512
    tokens = text + side * side
    h = bf16_round(randn(tokens * hidden, 1))
    q8, qs = O.quant_fp8_channel(randn(heads * 128 * hidden, 2, 0.02), heads * 128, hidden)
    qnorm = randn(128, 3, 0.1)
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(text, side, side), (16, 56, 56), 1e4)
    rope = we.Rope(graph.buffer(cos), graph.buffer(sin), pairs, tokens)
    hb, wq = graph.buffer(bf16(h)), we.Linear(graph.buffer(q8), "fp8", 1.0, heads * 128, hidden,
                                              chan_scale=graph.buffer(qs))
    q = we.linear(graph, hb, wq, tokens, x_dtype="bf16", y_dtype="f32")
    qn = we.norm(graph, q, graph.buffer(qnorm), tokens * heads, 128)
    qr = we.rotate(graph, qn, heads, rope)
    fused = we.qk_norm_rotate(graph, q, graph.buffer(qnorm), heads, rope)
    a = graph.read(qr, tokens * heads * 128 * 4, np.float32)
    b = graph.read(fused, tokens * heads * 128 * 4, np.float32)
    lin = O.matmul(h, O.FP8, q8, tokens, heads * 128, hidden, chan_scale=qs)
    want = O.rope(O.rmsnorm(lin.astype(np.float32), qnorm, None, None, 1e-5, 1.0).astype(np.float32), tokens, heads,
                  pairs, cos, sin)
    assert O.compare(a, want)["cosine"] > 0.99999 and np.max(np.abs(a - want)) < 1e-4
    assert np.max(np.abs(a - b)) < 1e-5
