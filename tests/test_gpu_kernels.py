"""GPU parity of the bandwidth kernels against the CPU oracle, through the C ABI.

Mirrors the reference's tests/gpu/fp8.test.ts, tests/gpu/rmsnorm.test.ts and tests/gpu/rope.test.ts
(same inputs, same tolerances), then adds bf16, the fused q/k norm + RoPE, the int4 decode, the
weight quantisers and the activation split (all bit-exact), at the reference's and BASELINE sizes.
"""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, lcg_floats, max_err, randn

pytestmark = pytest.mark.gpu

NAN_CODES = {0x7F, 0xFF}


# ---------------- unpackFp8: tests/gpu/fp8.test.ts ----------------
def test_unpack_fp8_decodes_every_byte_exactly(we, graph):  # fp8.test.ts:21-28
    allb = np.arange(256, dtype=np.uint8)
    gpu = we.kernels.unpack_fp8(graph, allb, 1.0)
    for b in range(256):
        if b not in NAN_CODES:
            assert gpu[b] == O.e4m3(b), hex(b)


def test_unpack_fp8_applies_the_per_tensor_scale(we, graph):  # fp8.test.ts:30-33
    s = 0.0018833705689758062
    gpu = we.kernels.unpack_fp8(graph, np.array([0x38, 0xC0, 0x7E], np.uint8), s)
    want = [np.float32(v) * np.float32(s) for v in (1, -2, 448)]
    assert gpu.tolist() == want


def test_unpack_fp8_ragged_lengths(we, graph):  # fp8.test.ts:35-37
    assert we.kernels.unpack_fp8(graph, np.array([0x38] * 4 + [0x40], np.uint8), 1.0).tolist() == [1, 1, 1, 1, 2]
    data = np.random.default_rng(0).integers(0, 256, 1000003, dtype=np.uint8)
    data[(data & 0x7F) == 0x7F] = 0
    gpu = we.kernels.unpack_fp8(graph, data, 0.5)
    assert np.array_equal(gpu, (O.e4m3_table()[data] * 0.5).astype(np.float32))


def test_unpack_fp8_to_bf16_is_exact(we, graph):
    data = np.random.default_rng(1).integers(0, 256, 4099, dtype=np.uint8)
    data[(data & 0x7F) == 0x7F] = 0
    mark = graph.mark()
    ib, ob = graph.buffer(data), graph.buffer(data.size * 2)
    we.kernels.unpack_fp8_bf16(graph, ib, data.size, ob)
    got = graph.read(ob, data.size * 2, np.uint16)
    assert np.array_equal(got, bf16(O.e4m3_table()[data].astype(np.float32)))
    graph.release(mark)


def test_int4_decode_is_bit_exact(we, graph):
    n, k = 96, 320
    w = randn(n * k, 3, 0.02)
    packed, scales = O.quant_int4_g64(w, n, k)
    mark = graph.mark()
    pb, sb, ob = graph.buffer(packed), graph.buffer(scales), graph.buffer(n * k * 2)
    we.kernels.unpack_int4(graph, pb, sb, n, k, ob)
    got = graph.read(ob, n * k * 2, np.uint16)
    nib = np.stack([packed & 0xF, packed >> 4], 1).reshape(n, k).astype(np.int32)
    q = np.where(nib >= 8, nib - 16, nib).astype(np.float32)
    s = scales.view(np.float16).astype(np.float32).reshape(n, k // 64)
    assert np.array_equal(got.reshape(n, k), bf16(q * np.repeat(s, 64, 1)))
    graph.release(mark)


# ---------------- quantisers (this build's conventions) ----------------
@pytest.mark.parametrize("n,k", [(64, 256), (37, 100), (3072, 3072)])
def test_quantize_fp8_per_channel_bit_exact(we, graph, n, k):
    w = randn(n * k, 7, 0.02)
    w[:k] = 0  # an all-zero channel (scale 1)
    q_ref, s_ref = O.quant_fp8_channel(w, n, k)
    mark = graph.mark()
    wb, qb, sb = graph.buffer(w), graph.buffer(n * k), graph.buffer(n * 4)
    we.kernels.quantize_fp8(graph, wb, n, k, qb, sb, per_channel=True)
    assert np.array_equal(graph.read(qb, n * k), q_ref)
    assert np.array_equal(graph.read(sb, n * 4, np.float32), s_ref)
    graph.release(mark)


def test_quantize_fp8_per_tensor_bit_exact(we, graph):
    n, k = 200, 160
    w = randn(n * k, 8, 0.05)
    q_ref, s_ref = O.quant_fp8_tensor(w, n, k)
    mark = graph.mark()
    wb, qb, sb = graph.buffer(w), graph.buffer(n * k), graph.buffer(4)
    we.kernels.quantize_fp8(graph, wb, n, k, qb, sb, per_channel=False)
    assert np.array_equal(graph.read(qb, n * k), q_ref)
    assert graph.read(sb, 4, np.float32)[0] == np.float32(s_ref)
    graph.release(mark)


@pytest.mark.parametrize("n,k", [(64, 256), (3072, 3072)])
def test_quantize_int4_bit_exact(we, graph, n, k):
    w = randn(n * k, 9, 0.02)
    w[64:128] = 0  # an all-zero group
    p_ref, s_ref = O.quant_int4_g64(w, n, k)
    mark = graph.mark()
    wb, pb, sb = graph.buffer(w), graph.buffer(n * k // 2), graph.buffer(n * k // 64 * 2)
    we.kernels.quantize_int4(graph, wb, n, k, pb, sb)
    assert np.array_equal(graph.read(pb, n * k // 2), p_ref)
    assert np.array_equal(graph.read(sb, n * k // 64 * 2, np.uint16), s_ref)
    graph.release(mark)


@pytest.mark.parametrize("m,k,terms", [(5, 512, 2), (64, 3072, 2), (33, 104, 2), (16, 3072, 1), (7, 37, 2)])
def test_activation_split_bit_exact(we, graph, m, k, terms):
    x = bf16_round(randn(m * k, 11, 2.0)).reshape(m, k)
    x[1] *= np.float32(300.0)
    x[2] *= np.float32(1e-3)
    x[3] = 0
    x[4] *= np.float32(1e-37)  # 2^-e above the largest float: the kernels' ldexpf path instead of a multiply
    x = bf16_round(x).reshape(m, k)
    mark = graph.mark()
    xb = graph.buffer(bf16(x))
    hb, lb, sb = graph.buffer(m * k), graph.buffer(m * k), graph.buffer(m * 4)
    we.kernels.quantize_act(graph, xb, m, k, hb, lb if terms > 1 else None, sb, terms=terms)
    hi, lo = graph.read(hb, m * k).reshape(m, k), graph.read(lb, m * k).reshape(m, k)
    rs = graph.read(sb, m * 4, np.float32)
    e4 = O.e4m3_table()
    for r in range(m):
        h, l_, e = O.act_split(x[r], terms)
        assert np.array_equal(hi[r], h), r
        if terms > 1:
            assert np.array_equal(lo[r], l_), r
        assert rs[r] == np.float32(2.0 ** e)
        if terms > 1:  # bf16 input: exact except below the smallest e4m3 step of the row scale
            back = (e4[hi[r]] + e4[lo[r]]) * 2.0 ** e
            assert np.all(np.abs(back - x[r]) <= 2.0 ** (e - 10))
    graph.release(mark)


# ---------------- rmsnorm: tests/gpu/rmsnorm.test.ts ----------------
def _centred(seed):
    r = O.lcg(seed)
    return lambda: r() - 0.5


def test_rmsnorm_krea_rows_with_modulation(we, graph):  # rmsnorm.test.ts:24-30
    r = _centred(1)
    d = 6144
    x = np.array([r() * 8 for _ in range(3 * d)], np.float32)
    w = np.array([r() * 0.2 for _ in range(d)], np.float32)
    sc = np.array([r() * 2 for _ in range(d)], np.float32)
    sh = np.array([r() * 2 for _ in range(d)], np.float32)
    gpu = we.kernels.rmsnorm_once(graph, x, w, scale=sc, shift=sh)
    assert max_err(gpu, O.rmsnorm(x, w, sc, sh, 1e-5, 1.0)) < 1e-5


def test_rmsnorm_plain_per_head(we, graph):  # rmsnorm.test.ts:32-39
    r = _centred(2)
    d = 128
    x = np.array([r() * 2 for _ in range(100 * d)], np.float32)
    w = np.array([r() * 2 for _ in range(d)], np.float32)
    gpu = we.kernels.rmsnorm_once(graph, x, w, offset=0.0)
    assert max_err(gpu, O.rmsnorm(x, w, None, None, 1e-5, 0.0)) < 1e-5


def test_rmsnorm_short_odd_rows(we, graph):  # rmsnorm.test.ts:41-47
    r = _centred(3)
    x = np.array([r() * 2 for _ in range(5 * 37)], np.float32)
    w = np.array([r() * 2 for _ in range(37)], np.float32)
    assert max_err(we.kernels.rmsnorm_once(graph, x, w), O.rmsnorm(x, w, None, None, 1e-5, 1.0)) < 1e-5
    with pytest.raises(ValueError, match="whole number of rows"):
        we.kernels.rmsnorm_once(graph, x[:-1], w)


def test_rmsnorm_block_size_bf16(we, graph):
    """Config 3's norm: 4608 x 3072 bf16 in and out; every row checked against float64."""
    rows, d = 4608, 3072
    x = bf16_round(randn(rows * d, 21, 1.0))
    w = randn(d, 22, 0.1)
    sc, sh = randn(d, 23, 0.3), randn(d, 24, 0.3)
    mark = graph.mark()
    xb, wb, scb, shb, ob = (graph.buffer(bf16(x)), graph.buffer(w), graph.buffer(sc), graph.buffer(sh),
                            graph.buffer(rows * d * 2))
    we.kernels.rmsnorm(graph, xb, wb, rows, d, ob, scb, shb, x_dtype="bf16", out_dtype="bf16")
    got = O.bf16_to_f32(graph.read(ob, rows * d * 2, np.uint16))
    want = O.rmsnorm(x, w, sc, sh, 1e-5, 1.0)
    # one bf16 rounding of the output: |err| <= 2^-8 |want| (+ fp32 noise)
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + 1e-5)
    graph.release(mark)


# ---------------- rope: tests/gpu/rope.test.ts ----------------
def test_rope_rotates_each_pair_by_its_tokens_angles(we, graph):  # rope.test.ts:5-23
    heads = 3
    pos = we.kernels.positions(2, 3, 4)
    tables = we.kernels.rope_tables(pos)
    x = lcg_floats(len(pos) * heads * 128, 1)
    gpu = we.kernels.rope_once(graph, x, heads, tables)
    cos, sin, pairs = tables
    want = O.rope(x, len(pos), heads, pairs, cos, sin)
    assert max_err(gpu, want) < 1e-6
    assert np.array_equal(gpu[: 2 * heads * 128], x[: 2 * heads * 128])  # text tokens unchanged


def test_rope_half_pairing_for_the_text_encoder(we, graph):  # rope.test.ts:25-42
    heads = 2
    pos = [[0], [1], [5], [40]]
    tables = we.kernels.rope_tables(pos, (128,), 5e6)
    x = lcg_floats(4 * heads * 128, 7)
    gpu = we.kernels.rope_once(graph, x, heads, tables, "half")
    cos, sin, pairs = tables
    assert max_err(gpu, O.rope(x, 4, heads, pairs, cos, sin, "half")) < 1e-5
    with pytest.raises(ValueError, match="does not match"):
        we.kernels.rope_once(graph, x[:-2], heads, tables)


@pytest.mark.parametrize("pairing", ["interleaved", "half"])
def test_rope_block_size_bf16(we, graph, pairing):
    """Config 3's q: 4608 tokens x 24 heads x 128, axes 16/56/56, theta 1e4, bf16."""
    tokens, heads = 512 + 64 * 64, 24
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(512, 64, 64), (16, 56, 56), 1e4)
    x = bf16_round(randn(tokens * heads * 128, 31))
    mark = graph.mark()
    xb, cb, sb, ob = graph.buffer(bf16(x)), graph.buffer(cos), graph.buffer(sin), graph.buffer(x.size * 2)
    we.kernels.rope_apply(graph, xb, cb, sb, tokens, heads, pairs, ob, pairing, x_dtype="bf16", out_dtype="bf16")
    got = O.bf16_to_f32(graph.read(ob, x.size * 2, np.uint16))
    want = O.rope(x, tokens, heads, pairs, cos, sin, pairing)
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + 1e-6)
    graph.release(mark)


# ---------------- fused q/k norm + RoPE (src/model/block.ts:53-56) ----------------
@pytest.mark.parametrize("pairing", ["interleaved", "half"])
def test_qknorm_rope_block_size_bf16(we, graph, pairing):
    """Config 3's q path in bf16: 4608 tokens x 24 heads x 128, axes 16/56/56, theta 1e4."""
    tokens, heads = 512 + 64 * 64, 24
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(512, 64, 64), (16, 56, 56), 1e4)
    x = bf16_round(randn(tokens * heads * 128, 41, 2.0))
    w = randn(128, 42, 0.1)
    mark = graph.mark()
    xb, wb, cb, sb, ob = (graph.buffer(bf16(x)), graph.buffer(w), graph.buffer(cos), graph.buffer(sin),
                          graph.buffer(x.size * 2))
    we.kernels.qknorm_rope(graph, xb, wb, cb, sb, tokens, heads, pairs, ob, pairing=pairing, x_dtype="bf16",
                           out_dtype="bf16")
    got = O.bf16_to_f32(graph.read(ob, x.size * 2, np.uint16))
    want = O.rope(O.rmsnorm(x, w, None, None, 1e-5, 1.0).astype(np.float32), tokens, heads, pairs, cos, sin, pairing)
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8 + 2e-5)
    graph.release(mark)


@pytest.mark.parametrize("head_dim,pairing,axes,heads", [
    (128, "interleaved", (32, 48, 48), 4), (128, "half", (32, 48, 48), 4), (128, "interleaved", (32, 48, 48), 3),
    (128, "half", (32, 48, 48), 3), (128, "interleaved", (32, 48, 48), 8), (128, "half", (32, 48, 48), 16),
    (64, "interleaved", (16, 24, 24), 4), (256, "interleaved", (64, 96, 96), 4), (96, "interleaved", (32, 32, 32), 4)])
def test_qknorm_rope_matches_norm_then_rotate(we, graph, head_dim, pairing, axes, heads):
    """With 3 heads an odd number of head rows; with 8 and 16 heads of 128 the kernel takes a token's 8 heads per
    warp step (its cos/sin loaded once for them)."""
    tokens = 2 + 5 * 7
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(2, 5, 7), axes, 1000.0)
    assert 2 * pairs == head_dim
    x = lcg_floats(tokens * heads * head_dim, 5, 3.0)
    w = lcg_floats(head_dim, 6, 0.5)
    mark = graph.mark()
    xb, wb, cb, sb, ob = (graph.buffer(x), graph.buffer(w), graph.buffer(cos), graph.buffer(sin),
                          graph.buffer(x.size * 4))
    we.kernels.qknorm_rope(graph, xb, wb, cb, sb, tokens, heads, pairs, ob, eps=1e-5, offset=1.0, pairing=pairing)
    got = graph.read(ob, x.size * 4, np.float32)
    normed = O.rmsnorm(x, w, None, None, 1e-5, 1.0)
    want = O.rope(normed.astype(np.float32), tokens, heads, pairs, cos, sin, pairing)
    assert max_err(got, want) < 2e-5
    graph.release(mark)
