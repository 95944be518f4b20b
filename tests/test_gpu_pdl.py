"""Programmatic dependent launch: the row kernels, GEMMs and flash attention may be placed on the SMs while the
kernel before them is finishing, and each waits (griddepcontrol.wait) before touching global memory. A kernel that
read or wrote too early would make a chain of dependent launches nondeterministic. Here a chain in which every
launch consumes the previous one's output (add + norm + split -> fp8 tensor-core GEMM -> add + norm + split -> ...,
and q/k norm + RoPE -> flash attention on the normalised rows) runs back to back with no host synchronisation, and
must equal, bit for bit, the same chain with the stream drained after every launch."""
import numpy as np
import pytest

from util import bf16, bf16_round, fast_fp8, randn

pytestmark = pytest.mark.gpu


def _chain(we, graph, m, d, steps, drain):
    K = we.kernels
    x0, r0 = randn(m * d, 91, 1.0), randn(m * d, 92, 0.1)
    w, sc, sh = randn(d, 93, 0.1), randn(d, 94, 0.3), randn(d, 95, 0.3)
    wq = fast_fp8(d * d, 96)
    cs = (np.abs(randn(d, 97, 0.002)) + np.float32(1e-4)).astype(np.float32)
    mark = graph.mark()
    xs = [graph.buffer(x0), graph.buffer(m * d * 4)]
    r = graph.buffer(r0)
    wb, scb, shb, wqb, csb = (graph.buffer(a) for a in (w, sc, sh, wq, cs))
    hi, lo, rs = graph.buffer(m * d), graph.buffer(m * d), graph.buffer(m * 4)
    for i in range(steps):
        xin, xout = xs[i % 2], xs[(i + 1) % 2]
        K.add_norm_split(graph, xin, r, xout, wb, m, d, hi, lo, rs, scale=scb, shift=shb)  # reads the GEMM's r
        if drain:
            graph.sync()
        K.gemm_fp8(graph, hi, lo, rs, wqb, r, m, d, d, chan_scale=csb, y_dtype="f32")  # overwrites r
        if drain:
            graph.sync()
    out = graph.read(xs[steps % 2], m * d * 4, np.float32).copy()
    planes = graph.read(hi, m * d).copy()
    graph.release(mark)
    return out, planes


def test_dependent_chain_equals_the_drained_chain(we, graph):
    got, got_hi = _chain(we, graph, 512, 3072, 20, drain=False)
    want, want_hi = _chain(we, graph, 512, 3072, 20, drain=True)
    assert np.isfinite(want).all()
    assert np.array_equal(got, want) and np.array_equal(got_hi, want_hi)
    assert graph.device_error() == 0


def test_attention_after_qk_norm_equals_the_drained_order(we, graph):
    K = we.kernels
    tokens, heads, dim = 700, 4, 128
    q, k, v = (bf16_round(randn(tokens * heads * dim, s, 1.0)) for s in (101, 102, 103))
    qn = randn(dim, 104, 0.1)
    cos, sin, pairs = K.rope_tables(K.positions(60, 20, 32), (16, 56, 56), 1e4)

    def run(drain):
        mark = graph.mark()
        qb, kb, vb = graph.buffer(bf16(q)), graph.buffer(bf16(k)), graph.buffer(bf16(v))
        qnb, cb, sb = graph.buffer(qn), graph.buffer(cos), graph.buffer(sin)
        ob = graph.buffer(tokens * heads * dim * 2)
        outs = []
        for _ in range(3):  # in place: each round normalises and rotates the previous round's q and k
            K.qknorm_rope(graph, qb, qnb, cb, sb, tokens, heads, pairs, qb, x_dtype="bf16", out_dtype="bf16")
            if drain:
                graph.sync()
            K.qknorm_rope(graph, kb, qnb, cb, sb, tokens, heads, pairs, kb, x_dtype="bf16", out_dtype="bf16")
            if drain:
                graph.sync()
            K.attention(graph, qb, kb, vb, tokens, heads, heads, dim, ob, dtype="bf16", out_dtype="bf16")
            if drain:
                graph.sync()
            outs.append(graph.read(ob, tokens * heads * dim * 2, np.uint16).copy())
        graph.release(mark)
        return outs

    for a, b in zip(run(False), run(True)):
        assert np.array_equal(a, b)
    assert graph.device_error() == 0
