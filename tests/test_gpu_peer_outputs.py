"""The peer outputs of sequence parallelism, on one GPU: the kernels that produce q, k and v can store each head's
rows straight into the memory of the rank that attends that head (we_gemm_fp8_desc.peer_*, we_qknorm_rope_peers).
Here every "rank" is a local buffer, so the test checks the address arithmetic and the values bit for bit against
the ordinary outputs: head h of token t lands in destination h // (heads / world) at row row0 + t, head h % (heads /
world) of its [world x tokens, heads / world, 128] block."""
import numpy as np
import pytest

from util import bf16, bf16_round, fast_fp8, randn

pytestmark = pytest.mark.gpu


def _heads_of(flat, tokens, heads):
    return flat.reshape(tokens, heads, 128)


@pytest.mark.parametrize("world,row0", [(2, 100), (4, 0)])
def test_gemm_peer_part_lands_at_the_owners_rows(we, graph, world, row0):
    K = we.kernels
    m, k, hq, hk = 100, 256, 4, 4
    n = (hq + 2 * hk) * 128
    x = bf16_round(randn(m * k, 61))
    w = fast_fp8(n * k, 62)
    cs = (np.abs(randn(n, 63, 0.004)) + np.float32(1e-3)).astype(np.float32)
    mark = graph.mark()
    xb, wb, csb = graph.buffer(bf16(x)), graph.buffer(w), graph.buffer(cs)
    hi, lo, rs = graph.buffer(m * k), graph.buffer(m * k), graph.buffer(m * 4)
    K.quantize_act(graph, xb, m, k, hi, lo, rs, terms=2)
    parts = [(graph.buffer(m * hq * 256), hq * 128), (graph.buffer(m * hk * 256), hk * 128),
             (graph.buffer(m * hk * 256), hk * 128)]
    K.gemm_fp8(graph, hi, lo, rs, wb, None, m, n, k, chan_scale=csb, y_dtype="bf16", parts=parts)
    want_v = _heads_of(graph.read(parts[2][0], m * hk * 256, np.uint16), m, hk)
    want_q = graph.read(parts[0][0], m * hq * 256, np.uint16).copy()
    hl, rows = hk // world, row0 + m
    dst = [graph.buffer(np.zeros(rows * hl * 128, np.uint16)) for _ in range(world)]
    parts2 = [(graph.buffer(m * hq * 256), hq * 128), (graph.buffer(m * hk * 256), hk * 128),
              (graph.buffer(m * hk * 256), hk * 128)]
    K.gemm_fp8(graph, hi, lo, rs, wb, None, m, n, k, chan_scale=csb, y_dtype="bf16", parts=parts2,
               peer=dict(dst=[d.ptr for d in dst], part=2, row0=row0))
    for o in range(world):
        got = graph.read(dst[o], rows * hl * 256, np.uint16).reshape(rows, hl, 128)
        assert np.array_equal(got[row0:], want_v[:, o * hl:(o + 1) * hl]), o
        assert not got[:row0].any()  # rows of the other ranks are not touched
    assert np.array_equal(graph.read(parts2[0][0], m * hq * 256, np.uint16), want_q)  # the local parts as before
    graph.release(mark)
    assert graph.device_error() == 0


@pytest.mark.parametrize("heads,world,pairing", [(8, 2, "interleaved"), (6, 3, "half"), (4, 4, "interleaved")])
def test_qknorm_rope_peers_equals_qknorm_rope_rearranged(we, graph, heads, world, pairing):
    K = we.kernels
    tokens = 90
    x = bf16_round(randn(tokens * heads * 128, 71, 2.0))
    wn = randn(128, 72, 0.1)
    cos, sin, pairs = K.rope_tables(K.positions(10, 8, 10), (16, 56, 56), 1e4)
    mark = graph.mark()
    xb, wb, cb, sb = graph.buffer(bf16(x)), graph.buffer(wn), graph.buffer(cos), graph.buffer(sin)
    out = graph.buffer(tokens * heads * 256)
    K.qknorm_rope(graph, xb, wb, cb, sb, tokens, heads, pairs, out, pairing=pairing, x_dtype="bf16",
                  out_dtype="bf16")
    want = _heads_of(graph.read(out, tokens * heads * 256, np.uint16), tokens, heads)
    hl, row0 = heads // world, 7
    rows = row0 + tokens
    dst = [graph.buffer(np.zeros(rows * hl * 128, np.uint16)) for _ in range(world)]
    K.qknorm_rope_peers(graph, xb, wb, cb, sb, tokens, heads, [d.ptr for d in dst], row0, pairing=pairing)
    for o in range(world):
        got = graph.read(dst[o], rows * hl * 256, np.uint16).reshape(rows, hl, 128)
        assert np.array_equal(got[row0:], want[:, o * hl:(o + 1) * hl]), o
        assert not got[:row0].any()
    graph.release(mark)
    assert graph.device_error() == 0


def test_peer_outputs_refuse_bad_layouts(we, graph):
    K = we.kernels
    mark = graph.mark()
    b = graph.buffer(1 << 16)
    with pytest.raises(we._lib.WeError, match="heads must split"):
        K.qknorm_rope_peers(graph, b, b, b, b, 4, 6, [b.ptr] * 4, 0)
    with pytest.raises(we._lib.WeError, match="peer output"):  # f32 output
        K.gemm_fp8(graph, b, None, b, b, b, 16, 256, 64, y_dtype="f32", peer=dict(dst=[b.ptr, b.ptr], row0=0))
    with pytest.raises(we._lib.WeError, match="peer output"):  # 256 channels do not split into heads over 4 ranks
        K.gemm_fp8(graph, b, None, b, b, b, 16, 256, 64, y_dtype="bf16", peer=dict(dst=[b.ptr] * 4, row0=0))
    graph.release(mark)
