"""The per-value ops, the GEMM-epilogue fusions, RMSNorm + split, and a whole block on the GPU.

Elementwise ops mirror tests/gpu/elementwise.test.ts (same tolerances). The block is checked against a
float64 restatement of tests/gpu/block.test.ts:26-100: in f32 on its tiny GQA config with the reference's
tolerance (cosine > 0.99999, relErr < 1e-4); in bf16 (fused B200 path: norm + split, fp8 tcgen05 GEMMs with
fused epilogues, q/k norm + RoPE, flash attention) on 128-wide heads with SwiGLU and GELU MLPs, where the
block's update (out - x) must reach cosine >= 0.9999 and max-abs-rel < 1e-2.
"""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, fast_fp8, lcg_floats, make_block, randn

pytestmark = pytest.mark.gpu


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v.astype(np.float64)))


def gelu(v):
    v = v.astype(np.float64)
    return 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))


def ew(we, graph, op, a, b=None, g=None, d=1, dtype="f32"):
    mark = graph.mark()
    try:
        conv = bf16 if dtype == "bf16" else (lambda z: np.asarray(z, np.float32))
        ab = graph.buffer(conv(a))
        bb = graph.buffer(conv(b)) if b is not None else None
        gb = graph.buffer(np.asarray(g, np.float32)) if g is not None else None
        out = we.ops.elementwise(graph, op, ab, bb, a.size, g=gb, d=d, dtype=dtype, out_dtype="f32")
        return graph.read(out, a.size * 4, np.float32).copy()
    finally:
        graph.release(mark)


def test_elementwise_ops_match_the_reference_formulas(we, graph):  # tests/gpu/elementwise.test.ts:15-37
    n, d = 1000, 40
    a, b = lcg_floats(n, 1, 8.0), lcg_floats(n, 2, 8.0)
    g = lcg_floats(d, 7, 1.0)
    af, bf = a.astype(np.float64), b.astype(np.float64)
    assert np.max(np.abs(ew(we, graph, "swiglu", a, b) - af * sigmoid(a) * bf)) < 1e-4
    assert np.max(np.abs(ew(we, graph, "sigmoid_gate", a, b) - af * sigmoid(b))) < 1e-5
    gi = g[np.arange(n) % d].astype(np.float64)
    assert np.max(np.abs(ew(we, graph, "gated_add", a, b, g=g, d=d) - (af + gi * bf))) < 1e-5
    assert np.max(np.abs(ew(we, graph, "add_bias", a, g=g, d=d) - (af + gi))) < 1e-5
    assert np.max(np.abs(ew(we, graph, "add", a, b) - (af + bf))) < 1e-5
    assert np.max(np.abs(ew(we, graph, "gelu_tanh", a) - gelu(a))) < 1e-5
    assert np.max(np.abs(ew(we, graph, "silu", a) - af * sigmoid(a))) < 1e-5
    # ragged length with bf16 inputs: the tail path and the 8-wide path agree
    x = bf16_round(randn(1003, 3, 4.0))
    y = bf16_round(randn(1003, 4, 4.0))
    assert np.max(np.abs(ew(we, graph, "swiglu", x, y, dtype="bf16") - x * sigmoid(x) * y)) < 1e-4


@pytest.mark.parametrize("rows,d,xdt", [(300, 3072, "bf16"), (300, 3072, "f32"), (64, 512, "f32"), (17, 136, "f32"),
                                        (5, 8192, "f32")])
def test_norm_split_equals_norm_then_split(we, graph, rows, d, xdt):
    x = randn(rows * d, 11, 2.0)
    if xdt == "bf16":
        x = bf16_round(x)
    w, sc, sh = randn(d, 12, 0.1), randn(d, 13, 0.3), randn(d, 14, 0.3)
    mark = graph.mark()
    xb = graph.buffer(bf16(x) if xdt == "bf16" else x)
    wb, scb, shb = graph.buffer(w), graph.buffer(sc), graph.buffer(sh)
    h = graph.buffer(rows * d * 2)
    we.kernels.rmsnorm(graph, xb, wb, rows, d, h, scb, shb, x_dtype=xdt, out_dtype="bf16")
    a = [graph.buffer(rows * d), graph.buffer(rows * d), graph.buffer(rows * 4)]
    we.kernels.quantize_act(graph, h, rows, d, *a, terms=2)
    b = [graph.buffer(rows * d), graph.buffer(rows * d), graph.buffer(rows * 4)]
    we.kernels.norm_split(graph, xb, wb, rows, d, *b, scale=scb, shift=shb, x_dtype=xdt)
    planes = [graph.read(buf, nb).copy() for buf, nb in zip(a + b, (rows * d, rows * d, rows * 4) * 2)]
    graph.release(mark)
    e4 = O.e4m3_table()
    recon = [(e4[hi] + e4[lo]).reshape(rows, d) * rs.view(np.float32)[:, None]
             for hi, lo, rs in (planes[:3], planes[3:])]
    # the two paths sum the row's squares in different orders: a rare 1-ulp bf16 difference, and when that moves
    # the row maximum across a power of two the scale differs and the smallest values round in e4m3's subnormal
    # range (absolute step 2^-9 of the scale, about 2^-17 of the row maximum)
    diff = np.abs(recon[0] - recon[1])
    rowmax = np.abs(recon[0]).max(axis=1, keepdims=True)
    assert np.all(diff <= np.abs(recon[0]) * 2.0 ** -7 + rowmax * 2.0 ** -16)
    assert np.mean(diff == 0) > 0.999


@pytest.mark.parametrize("path", ["tc", "simt"])
def test_gemm_epilogue_fusions(we, graph, path):
    m, n, k = 150, 264, 256
    x = bf16_round(randn(m * k, 21))
    w = fast_fp8(n * k, 22)
    cs = (np.abs(randn(n, 23, 0.004)) + np.float32(1e-3)).astype(np.float32)
    aux = bf16_round(randn(m * n, 24, 2.0))
    gate = randn(n, 25)
    start = randn(m * n, 26)
    base = O.matmul(x, O.FP8, w, m, n, k, chan_scale=cs).reshape(m, n)
    xd = "bf16" if path == "tc" else "f32"
    mark = graph.mark()
    xb = graph.buffer(bf16(x) if path == "tc" else x)
    wb, csb, auxb, gb = graph.buffer(w), graph.buffer(cs), graph.buffer(bf16(aux)), graph.buffer(gate)
    cases = {
        "gelu": (dict(act="gelu_tanh"), gelu(base)),
        "sigmoid_gate": (dict(aux_op="sigmoid_gate", aux=auxb, aux_dtype="bf16"),
                         aux.reshape(m, n) * sigmoid(base)),
        "swiglu": (dict(aux_op="swiglu", aux=auxb, aux_dtype="bf16"),
                   aux.reshape(m, n) * sigmoid(aux.reshape(m, n)) * base),
    }
    for name, (epi, want) in cases.items():
        yb = graph.buffer(m * n * 4)
        before = graph.stats["tcGemms"]
        we.kernels.matmul(graph, xb, wb, yb, m, n, k, 1.0, x_dtype=xd, w_dtype="fp8", chan_scale=csb,
                          force_simt=path == "simt", **epi)
        assert (graph.stats["tcGemms"] > before) == (path == "tc")
        got = graph.read(yb, m * n * 4, np.float32).reshape(m, n)
        assert O.rel_error(got, want) < 1e-5, name
    # gated residual: y = start + gate[col] * (x W^T)
    yb = graph.buffer(start)
    we.kernels.matmul(graph, xb, wb, yb, m, n, k, 1.0, x_dtype=xd, w_dtype="fp8", chan_scale=csb,
                      force_simt=path == "simt", accumulate=True, gate=gb)
    got = graph.read(yb, m * n * 4, np.float32).reshape(m, n)
    assert O.rel_error(got, start.reshape(m, n) + gate.astype(np.float64) * base) < 1e-5
    graph.release(mark)


def test_block_f32_matches_the_float64_block(we, graph):  # tests/gpu/block.test.ts:102-136
    cfg = we.blocks.BlockConfig(hidden=64, mlp=96, heads=4, kv_heads=2, head_dim=16)
    tokens = 4 + 3 * 4
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(4, 3, 4), (4, 6, 6), 1000.0)
    host, bw = make_block(we, graph, cfg, 100)
    x, temb = randn(tokens * cfg.hidden, 1, 1.0), randn(6 * cfg.hidden, 2, 0.3)
    want = O.block_reference(x.reshape(tokens, -1), host, vars(cfg), temb, cos, sin)
    mark = graph.mark()
    rope = we.Rope(graph.buffer(cos), graph.buffer(sin), pairs, tokens)
    out = we.blocks.block(graph, bw, cfg, graph.buffer(x), graph.buffer(temb), rope, dtype="f32")
    got = graph.read(out, tokens * cfg.hidden * 4, np.float32)
    graph.release(mark)
    c = O.compare(got, want.ravel())
    assert c["cosine"] > 0.99999 and c["relativeError"] < 1e-4, c


@pytest.mark.parametrize("mlp_act,kv_heads,per_channel", [("swiglu", 2, False), ("gelu", 4, True)])
def test_block_bf16_fused_path(we, graph, mlp_act, kv_heads, per_channel):
    cfg = we.blocks.BlockConfig(hidden=512, mlp=2048, heads=4, kv_heads=kv_heads, head_dim=128, mlp_act=mlp_act,
                                attn_gate=mlp_act == "swiglu")
    text, side = 16, 20
    tokens = text + side * side
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(text, side, side), (32, 48, 48), 1e4)
    host, bw = make_block(we, graph, cfg, 200, per_channel)
    x, temb = randn(tokens * cfg.hidden, 3, 1.0), randn(6 * cfg.hidden, 4, 0.3)
    want = O.block_reference(x.reshape(tokens, -1), host, vars(cfg), temb, cos, sin)
    mark = graph.mark()
    rope = we.Rope(graph.buffer(cos), graph.buffer(sin), pairs, tokens)
    out = we.blocks.block(graph, bw, cfg, graph.buffer(x), graph.buffer(temb), rope, dtype="bf16")
    got = graph.read(out, tokens * cfg.hidden * 4, np.float32).reshape(tokens, -1)
    assert graph.device_error() == 0
    graph.release(mark)
    delta, wdelta = got - x.reshape(tokens, -1), want - x.reshape(tokens, -1)
    c = O.compare(delta.ravel(), wdelta.ravel())
    rel = float(np.max(np.abs(delta - wdelta)) / np.max(np.abs(wdelta)))
    assert c["cosine"] >= 0.9999 and rel < 1e-2, (c, rel)


@pytest.mark.parametrize("pair", ["0", "2"], ids=["1sm", "pair"])
@pytest.mark.parametrize("m", [150, 1000])
def test_gemm_split_output(we, graph, monkeypatch, pair, m):
    """we_gemm_fp8 with a split output writes channels [0, 512), [512, 768), [768, 1024) (and [0, 384), [384, 640),
    [640, 1024): boundaries inside a 256-channel pair tile) to three buffers with rows as wide as each part, bit for
    bit the columns of the unsplit output; bad splits are refused."""
    monkeypatch.setenv("WE_TC_2SM", pair)
    n, k = 1024, 256
    x = bf16_round(randn(m * k, 31))
    w = fast_fp8(n * k, 32)
    cs = (np.abs(randn(n, 33, 0.004)) + np.float32(1e-3)).astype(np.float32)
    bias = randn(n, 34)
    mark = graph.mark()
    hi, lo, rs = graph.buffer(m * k), graph.buffer(m * k), graph.buffer(m * 4)
    we.kernels.quantize_act(graph, graph.buffer(bf16(x)), m, k, hi, lo, rs, terms=2)
    wb, csb, bb = graph.buffer(w), graph.buffer(cs), graph.buffer(bias)
    whole = graph.buffer(m * n * 2)
    we.kernels.gemm_fp8(graph, hi, lo, rs, wb, whole, m, n, k, chan_scale=csb, bias=bb, y_dtype="bf16")
    want = graph.read(whole, m * n * 2, np.uint16).reshape(m, n)
    for widths in ((512, 256, 256), (384, 256, 384)):
        parts = [(graph.buffer(m * wd * 2), wd) for wd in widths]
        we.kernels.gemm_fp8(graph, hi, lo, rs, wb, None, m, n, k, chan_scale=csb, bias=bb, y_dtype="bf16",
                            parts=parts)
        c0 = 0
        for buf, wd in parts:
            got = graph.read(buf, m * wd * 2, np.uint16).reshape(m, wd)
            assert np.array_equal(got, want[:, c0:c0 + wd])
            c0 += wd
    # widths that do not sum to n, and a boundary inside an epilogue warp's 32 channels
    for bad in ([(parts[0][0], 400), (parts[1][0], 624)], [(parts[0][0], 512), (parts[1][0], 256)]):
        with pytest.raises(we._lib.WeError, match="split output"):
            we.kernels.gemm_fp8(graph, hi, lo, rs, wb, None, m, n, k, chan_scale=csb, y_dtype="bf16", parts=bad)
    assert graph.device_error() == 0
    graph.release(mark)


@pytest.mark.parametrize("mlp_act,kv_heads,per_channel", [("swiglu", 2, False), ("gelu", 4, True)])
def test_fused_qkv_equals_three_gemms(we, graph, mlp_act, kv_heads, per_channel):
    """The block with wq, wk and wv fused into one GEMM (split epilogue, fuse_qkv) gives the same bits as with
    three GEMMs: each output channel's dot product and scale are the same."""
    cfg = we.blocks.BlockConfig(hidden=512, mlp=2048, heads=4, kv_heads=kv_heads, head_dim=128, mlp_act=mlp_act,
                                attn_gate=mlp_act == "swiglu")
    text, side = 16, 20
    tokens = text + side * side
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(text, side, side), (32, 48, 48), 1e4)
    _, bw = make_block(we, graph, cfg, 210, per_channel, fuse=False)
    x, temb = randn(tokens * cfg.hidden, 5, 1.0), randn(6 * cfg.hidden, 6, 0.3)
    rope = we.Rope(graph.buffer(cos), graph.buffer(sin), pairs, tokens)
    xb, tb = graph.buffer(x), graph.buffer(temb)

    def run():
        mark = graph.mark()
        out = we.blocks.block(graph, bw, cfg, xb, tb, rope, dtype="bf16")
        got = graph.read(out, tokens * cfg.hidden * 4, np.float32).copy()
        graph.release(mark)
        return got

    three = run()
    assert bw.wqkv is None
    we.blocks.fuse_qkv(graph, bw)
    assert bw.wqkv is not None and bw.wqkv.n == (cfg.heads + 2 * kv_heads) * 128
    fused = run()
    assert np.array_equal(three, fused)
    assert graph.device_error() == 0


@pytest.mark.parametrize("rows,d", [(300, 3072), (33, 512), (7, 64)])
def test_add_norm_split_equals_add_then_norm_split(we, graph, rows, d):
    """we_add_norm_split: xo = x + r exactly, and the planes of norm(xo) exactly as we_norm_split makes them."""
    x, r = randn(rows * d, 41, 2.0), randn(rows * d, 42, 0.5)
    w, sc, sh = randn(d, 43, 0.1), randn(d, 44, 0.3), randn(d, 45, 0.3)
    mark = graph.mark()
    xb, rb, wb, scb, shb = (graph.buffer(a) for a in (x, r, w, sc, sh))
    xo = graph.buffer(rows * d * 4)
    a = [graph.buffer(rows * d), graph.buffer(rows * d), graph.buffer(rows * 4)]
    we.kernels.add_norm_split(graph, xb, rb, xo, wb, rows, d, *a, scale=scb, shift=shb)
    xs = graph.buffer((x + r).astype(np.float32))
    b = [graph.buffer(rows * d), graph.buffer(rows * d), graph.buffer(rows * 4)]
    we.kernels.norm_split(graph, xs, wb, rows, d, *b, scale=scb, shift=shb, x_dtype="f32")
    got_x = graph.read(xo, rows * d * 4, np.float32).copy()
    planes = [graph.read(buf, nb).copy() for buf, nb in zip(a + b, (rows * d, rows * d, rows * 4) * 2)]
    graph.release(mark)
    assert np.array_equal(got_x, (x + r).astype(np.float32))
    for u, v in zip(planes[:3], planes[3:]):  # both run the same CTA-per-row kernel at every width: identical bits
        assert np.array_equal(u, v)
