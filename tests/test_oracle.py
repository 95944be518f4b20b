"""The CPU oracle against the reference's known-answer tests and the committed golden vectors.

These pin the oracle before any GPU result is compared with it. Known-answer values quote
the reference test they come from (file:line in dotstories/web-engine).
"""
import hashlib
import json
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "golden.json")))


def sha(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


# ---------- decoders: tests/fp8.test.ts ----------
@pytest.mark.parametrize("byte,value", [(0x00, 0), (0x38, 1), (0xC0, -2), (0x7E, 448), (0x01, 2 ** -9),
                                        (0x08, 2 ** -6), (0x3C, 1.5)])
def test_e4m3_known_answers(byte, value):  # tests/fp8.test.ts:5-13
    assert O.e4m3(byte) == value


def test_e4m3_negative_zero_and_nan():  # tests/fp8.test.ts:15-19
    assert math.copysign(1, O.e4m3(0x80)) == -1 and O.e4m3(0x80) == 0
    assert math.isnan(O.e4m3(0x7F)) and math.isnan(O.e4m3(0xFF))


def test_e4m3_all_bytes_match_torch():
    for b, v in enumerate(GOLDEN["e4m3"]):
        got = O.e4m3(b)
        assert (v is None and math.isnan(got)) or got == v, hex(b)


@pytest.mark.parametrize("byte,value", [(0x00, 0), (0x3C, 1), (0x7B, 57344), (0x01, 2 ** -16), (0xC0, -2)])
def test_e5m2_known_answers(byte, value):  # tests/fp8.test.ts:22-29
    assert O.e5m2(byte) == value


def test_e5m2_all_bytes_match_torch():
    for b, v in enumerate(GOLDEN["e5m2"]):
        got = O.e5m2(b)
        if v is None:
            assert math.isnan(got)
        else:
            assert got == v, hex(b)


def test_f16_bf16_decode_match_torch():
    for c, v in zip(GOLDEN["f16"]["codes"], GOLDEN["f16"]["values"]):
        assert O.f16(c) == v, hex(c)
    for c, v in zip(GOLDEN["bf16"]["codes"], GOLDEN["bf16"]["values"]):
        assert float(O.bf16_to_f32([c])[0]) == v, hex(c)


def test_to_float32():  # tests/fp8.test.ts:37-49
    le = lambda *w: np.array(w, dtype=np.uint16).tobytes()  # noqa: E731
    assert O.to_float32("F32", np.array([1.5, -2], np.float32).tobytes()).tolist() == [1.5, -2]
    assert O.to_float32("BF16", le(0x3F80, 0xC000)).tolist() == [1, -2]
    assert O.to_float32("F16", le(0x3C00, 0xC000, 0x0001, 0x7C00)).tolist() == [1, -2, 2 ** -24, math.inf]
    assert O.to_float32("F8_E4M3", bytes([0x38, 0x7E])).tolist() == [1, 448]
    assert O.to_float32("F8_E5M2", bytes([0x3C])).tolist() == [1]
    with pytest.raises(ValueError, match="I64"):
        O.to_float32("I64", bytes(8))


# ---------- encoders (round to nearest even) ----------
def test_e4m3_encode_matches_torch():
    g = GOLDEN["e4m3_encode"]
    got = [O.f32_to_e4m3(v) for v in g["in"]]
    assert got == g["out"]


def test_e4m3_encode_saturates():
    assert O.f32_to_e4m3(464.0) == 0x7E and O.f32_to_e4m3(1e9) == 0x7E and O.f32_to_e4m3(-1e9) == 0xFE
    assert O.f32_to_e4m3(float("nan")) == 0x7F


def test_bf16_f16_encode_match_torch():
    g = GOLDEN["bf16_encode"]
    assert O.bf16_bits(np.array(g["in"], np.float32)).tolist() == g["out"]
    g = GOLDEN["f16_encode"]
    assert [O.f32_to_f16(v) for v in g["in"]] == g["out"]


# ---------- noise: tests/noise.test.ts ----------
def test_mt19937_known_answer():  # tests/noise.test.ts:17-22
    mt = O.MT19937(5489)
    last = 0
    for _ in range(10000):
        last = mt.next()
    assert last == 4123659995


def test_mt19937_keeps_low_32_bits():  # tests/noise.test.ts:24-26
    assert O.MT19937(2 ** 32 + 7).next() == O.MT19937(7).next()


def test_torch_randn_known_answers():  # tests/noise.test.ts:31-45
    r4 = lambda a: [round(float(v) * 1e4) / 1e4 for v in a]  # noqa: E731
    assert r4(O.torch_randn(6, 0)) == [1.541, -0.2934, -2.1788, 0.5684, -1.0845, -1.3986]
    assert r4(O.torch_randn(3, 42)) == [0.3367, 0.1288, 0.2345]
    assert r4(O.torch_randn(16, 0)) == [-1.1258, -1.1524, -0.2506, -0.4339, 0.8487, 0.692, -0.316, -2.1152,
                                        0.3223, -1.2633, 0.35, 0.3081, 0.1198, 1.2377, 1.1168, -0.2473]


def test_torch_randn_matches_torch_golden():  # tests/noise.test.ts:47-52 + real torch
    for c in GOLDEN["torch_randn"]:
        a = O.torch_randn(c["n"], c["seed"])
        for i, v in c["values"].items():
            assert abs(float(a[int(i)]) - v) < 1e-6, (c["n"], c["seed"], i)


def test_torch_randn_big_latent_is_standard_normal():  # tests/noise.test.ts:54-60
    a = O.torch_randn(16 * 128 * 128, 54460995).astype(np.float64)
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1) < 0.01


# ---------- matmul: tests/gpu/matmul.test.ts ----------
def lcg_data(m, n, k, seed):
    """tests/gpu/matmul.test.ts:14-23"""
    r = O.lcg(seed)
    x = np.array([r() * 2 - 1 for _ in range(m * k)], dtype=np.float32)
    w = []
    for _ in range(n * k):
        b = math.floor(r() * 256)
        w.append(b - 1 if (b & 0x7F) == 0x7F else b)
    return x, np.array(w, dtype=np.uint8)


@pytest.mark.parametrize("case", GOLDEN["matmul"], ids=lambda c: f"{c['m']}x{c['n']}x{c['k']}")
def test_matmul_matches_golden(case):
    m, n, k = case["m"], case["n"], case["k"]
    x, w = lcg_data(m, n, k, case["seed"])
    assert sha(x) == case["x_sha256"] and sha(w) == case["w_sha256"]
    y = O.matmul(x, O.FP8, w, m, n, k, scale=case["scale"])
    for i, v in case["y_at"].items():
        assert abs(y[int(i)] - v) <= 1e-12 * max(1.0, abs(v))
    assert abs(y.sum() - case["y_sum"]) <= 1e-9 * case["y_abs_sum"]


def test_matmul_layouts_split_and_accumulate():
    m, n, k = 5, 12, 200
    x, w = lcg_data(m, n, k, 3)
    full = O.matmul(x, O.FP8, w, m, n, k, scale=0.5)
    parts = O.matmul(x, O.FP8, w, m, n, k, scale=0.5, k_split=3)  # slices of 80, 80, 40
    assert parts.size == 3 * m * n
    np.testing.assert_allclose(parts.reshape(3, -1).sum(0), full, rtol=0, atol=1e-12)
    assert abs(parts[0] - full[0]) > 1e-3
    start = np.arange(m * n, dtype=np.float64)
    acc = O.matmul(x, O.FP8, w, m, n, k, scale=0.5, accumulate=True, y=start.copy())
    np.testing.assert_allclose(acc, full + start, rtol=0, atol=1e-12)
    # strided head pick (tests/gpu/matmul.test.ts:95-110): Q.K^T of head 2 with kv head 1
    tokens, heads, kvh, dim = 20, 4, 2, 128
    r = O.lcg(3)
    q = np.array([r() * 2 - 1 for _ in range(tokens * heads * dim)], np.float32)
    r = O.lcg(4)
    kk = np.array([r() * 2 - 1 for _ in range(tokens * kvh * dim)], np.float32)
    s = O.matmul(q, O.F32, kk, tokens, tokens, dim, x_stride=heads * dim, x_offset=2 * dim, w_stride=kvh * dim,
                 w_offset=dim, y_stride=24, y_len=tokens * 24)
    want = q.reshape(tokens, heads, dim)[:, 2].astype(np.float64) @ kk.reshape(tokens, kvh, dim)[:, 1].T
    np.testing.assert_allclose(s.reshape(tokens, 24)[:, :tokens], want, rtol=0, atol=1e-12)


def test_ksplit_for_known_answers():  # tests/gpu/matmul.test.ts:151-156
    assert O.ksplit_for(1088, 64, 6144) == 24
    assert O.ksplit_for(4160, 64, 16384) == 8
    assert O.ksplit_for(4160, 6144, 6144) == 1
    assert O.ksplit_for(5, 12, 16) == 1


def test_compare_and_rel_error():  # src/model/compare.ts:2-17
    a = np.array([1, 2, 3], np.float32)
    b = np.array([1, 2, 3.5])
    c = O.compare(a, b)
    assert c["maxError"] == 0.5
    assert abs(c["relativeError"] - 0.5 / math.sqrt(1 + 4 + 12.25)) < 1e-15
    assert abs(O.rel_error(a, b) - 0.5 / 3.5) < 1e-15


# ---------- rmsnorm: tests/gpu/rmsnorm.test.ts ----------
@pytest.mark.parametrize("case", GOLDEN["rmsnorm"], ids=lambda c: f"d{c['d']}")
def test_rmsnorm_matches_golden(case):
    r = O.lcg(case["seed"])
    rr = lambda: r() - 0.5  # noqa: E731
    rows, d = case["rows"], case["d"]
    if case["mod"]:
        x = np.array([rr() * 8 for _ in range(rows * d)], np.float32)
        w = np.array([rr() * 0.2 for _ in range(d)], np.float32)
        sc = np.array([rr() * 2 for _ in range(d)], np.float32)
        sh = np.array([rr() * 2 for _ in range(d)], np.float32)
    else:
        x = np.array([rr() * 2 for _ in range(rows * d)], np.float32)
        w = np.array([rr() * 2 for _ in range(d)], np.float32)
        sc = sh = None
    assert sha(x) == case["x_sha256"]
    y = O.rmsnorm(x, w, sc, sh, eps=1e-5, offset=case["offset"])
    for i, v in case["y_at"].items():
        assert abs(y[int(i)] - v) <= 1e-12 * max(1, abs(v))
    assert abs(y.sum() - case["y_sum"]) <= 1e-9 * np.abs(y).sum()


# ---------- rope: tests/rope.test.ts ----------
def test_positions_known_answer():  # tests/rope.test.ts:4-16
    assert O.positions(2, 2, 3).tolist() == [[0, 0, 0], [0, 0, 0], [0, 0, 0], [0, 0, 1], [0, 0, 2], [0, 1, 0],
                                             [0, 1, 1], [0, 1, 2]]


def test_rope_tables_known_answers():  # tests/rope.test.ts:19-38
    cos, sin, pairs = O.rope_tables([[0, 0, 0]])
    assert pairs == 64 and cos.tolist() == [1] * 64 and sin.tolist() == [0] * 64
    cos, sin, _ = O.rope_tables([[0, 3, 5]], [32, 48, 48], 1000)
    ang = lambda p, j, dim: p * 1000 ** (-(2 * j) / dim)  # noqa: E731
    assert sin[0] == 0
    assert abs(cos[16] - math.cos(ang(3, 0, 48))) < 5e-7
    assert abs(sin[16 + 5] - math.sin(ang(3, 5, 48))) < 5e-7
    assert abs(sin[40 + 23] - math.sin(ang(5, 23, 48))) < 5e-7
    with pytest.raises(ValueError, match="even"):
        O.rope_tables([[0, 0, 0]], [31, 48, 49])


def test_rope_tables_match_golden():
    for c in GOLDEN["rope_tables"]:
        cos, sin, _ = O.rope_tables(c["pos"], c["axes"], c["theta"])
        assert cos.tolist() == c["cos"] and sin.tolist() == c["sin"]


def test_rope_rotation_formulas():  # tests/gpu/rope.test.ts:14-21 and :33-40
    heads = 3
    pos = O.positions(2, 3, 4)
    cos, sin, pairs = O.rope_tables(pos)
    r = O.lcg(1)
    x = np.array([r() * 2 - 1 for _ in range(len(pos) * heads * 128)], np.float32)
    y = O.rope(x, len(pos), heads, pairs, cos, sin).reshape(len(pos), heads, 64, 2)
    xv = x.astype(np.float64).reshape(len(pos), heads, 64, 2)
    c = cos.reshape(len(pos), 1, 64).astype(np.float64)
    s = sin.reshape(len(pos), 1, 64).astype(np.float64)
    np.testing.assert_allclose(y[..., 0], xv[..., 0] * c - xv[..., 1] * s, atol=1e-15)
    np.testing.assert_allclose(y[..., 1], xv[..., 1] * c + xv[..., 0] * s, atol=1e-15)
    assert (y.ravel()[: 2 * heads * 128] == x[: 2 * heads * 128]).all()  # text tokens unchanged
    yh = O.rope(x, len(pos), heads, pairs, cos, sin, "half").reshape(len(pos), heads, 128)
    xh = x.astype(np.float64).reshape(len(pos), heads, 128)
    np.testing.assert_allclose(yh[..., :64], xh[..., :64] * c - xh[..., 64:] * s, atol=1e-15)


# ---------- this build's quantisers against their torch restatement ----------
def test_quant_fp8_channel_matches_torch():
    g = GOLDEN["quant_fp8_channel"]
    w = lcg_floats(g["n"] * g["k"], g["seed"], g["std"])
    assert sha(w) == g["w_sha256"]
    q, s = O.quant_fp8_channel(w, g["n"], g["k"])
    assert s.tolist() == pytest.approx(g["scales"], rel=0, abs=0)
    assert sha(q) == g["q_sha256"]


def test_quant_int4_g64_matches_torch():
    g = GOLDEN["quant_int4_g64"]
    n, k = g["n"], g["k"]
    w = lcg_floats(n * k, g["seed"], g["std"])
    packed, scales = O.quant_int4_g64(w, n, k)
    assert [int(v) - 65536 if v > 32767 else int(v) for v in scales] == g["scales"]
    assert sha(packed) == g["packed_sha256"]
    op = _int4_operands(packed, scales, n, k)
    assert sha(op) == g["operand_sha256"]


def lcg_floats(n, seed, size):
    r = O.lcg(seed)
    return np.array([(r() * 2 - 1) * size for _ in range(n)], np.float32)


def _int4_operands(packed, scales, n, k):
    nib = np.stack([packed & 0xF, packed >> 4], axis=1).reshape(n, k).astype(np.int32)
    q = np.where(nib >= 8, nib - 16, nib).astype(np.float32)
    s = scales.view(np.float16).astype(np.float32).reshape(n, k // 64)
    return O.bf16_round(q * np.repeat(s, 64, axis=1))


def test_act_split_matches_torch_and_is_exact():
    g = GOLDEN["act_split"]
    # the same rows as make_golden.py: LCG(5) * 3 rounded to bf16, rows 1-3 rescaled in float32
    base = O.bf16_round(lcg_floats(4 * 512, 5, 3.0)).reshape(4, 512)
    rows = [base[0], base[1] * np.float32(300.0), base[2] * np.float32(1e-3), np.zeros(512, np.float32)]
    for row, want in zip(rows, g["rows_out"]):
        hi, lo, e = O.act_split(row, 2)
        assert e == want["e"] and sha(hi) == want["hi_sha256"] and sha(lo) == want["lo_sha256"]
        e4 = O.e4m3_table()
        back = (e4[hi] + e4[lo]) * 2.0 ** e
        assert want["exact"] == bool((back == row.astype(np.float64)).all())
