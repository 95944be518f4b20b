"""ctypes + numpy view of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and by the
CPU-baseline leg of ``bench.py``. It is the checker, never the thing measured or shipped.
Each wrapper restates a reference function; the C source cites file:line for each.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

F32, BF16, FP8, INT4G64 = 0, 1, 2, 3


def build() -> str:
    """Compile the oracle (gcc + OpenMP) in place; returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load() -> C.CDLL:
    if not os.path.exists(_LIB_PATH):
        build()
    lib = C.CDLL(_LIB_PATH)
    p = C.c_void_p
    lib.or_e4m3.restype = C.c_double
    lib.or_e4m3.argtypes = [C.c_uint8]
    lib.or_e5m2.restype = C.c_double
    lib.or_e5m2.argtypes = [C.c_uint8]
    lib.or_f16.restype = C.c_double
    lib.or_f16.argtypes = [C.c_uint16]
    lib.or_f32_to_bf16.restype = C.c_uint16
    lib.or_f32_to_bf16.argtypes = [C.c_float]
    lib.or_f32_to_f16.restype = C.c_uint16
    lib.or_f32_to_f16.argtypes = [C.c_float]
    lib.or_f32_to_e4m3.restype = C.c_uint8
    lib.or_f32_to_e4m3.argtypes = [C.c_float]
    lib.or_to_float32.restype = C.c_long
    lib.or_to_float32.argtypes = [C.c_int, p, C.c_size_t, p]
    lib.or_mt_seed.argtypes = [p, C.c_uint64]
    lib.or_mt_next.restype = C.c_uint32
    lib.or_mt_next.argtypes = [p]
    lib.or_torch_randn.argtypes = [C.c_size_t, C.c_uint64, p]
    lib.or_matmul.argtypes = [p, C.c_int, p, C.c_double, p, p, p, p]
    lib.or_matmul_mt.argtypes = [p, C.c_int, p, C.c_double, p, p, p, p, C.c_int]
    lib.or_ksplit_for.restype = C.c_long
    lib.or_ksplit_for.argtypes = [C.c_long] * 3
    lib.or_rel_error.restype = C.c_double
    lib.or_rel_error.argtypes = [p, p, C.c_size_t]
    lib.or_compare.argtypes = [p, p, C.c_size_t, p, p, p]
    lib.or_quant_fp8_channel.argtypes = [p, C.c_long, C.c_long, p, p]
    lib.or_quant_fp8_tensor.restype = C.c_float
    lib.or_quant_fp8_tensor.argtypes = [p, C.c_long, C.c_long, p]
    lib.or_quant_int4_g64.argtypes = [p, C.c_long, C.c_long, p, p]
    lib.or_act_split.argtypes = [p, C.c_long, C.c_int, p, p, p]
    lib.or_rmsnorm.argtypes = [p, p, p, p, C.c_long, C.c_long, C.c_float, C.c_float, p]
    lib.or_positions.argtypes = [C.c_long, C.c_long, C.c_long, p]
    lib.or_rope_tables.restype = C.c_long
    lib.or_rope_tables.argtypes = [p, C.c_long, C.c_int, p, C.c_double, p, p]
    lib.or_rope.argtypes = [p, C.c_long, C.c_long, C.c_long, p, p, C.c_int, p]
    lib.or_attention.argtypes = [p, p, p, C.c_long, C.c_long, C.c_long, C.c_long, C.c_int, p]
    return lib


lib = _load()


class MMShape(C.Structure):
    _fields_ = [(n, C.c_long) for n in (
        "m", "n", "k", "x_stride", "w_stride", "y_stride", "x_offset", "w_offset", "y_offset", "k_split")] + [
        ("accumulate", C.c_int)]


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return None if a is None else np.ascontiguousarray(a, dtype=dtype)


# ---- decoders ----
def e4m3(b: int) -> float:
    return lib.or_e4m3(b)


def e5m2(b: int) -> float:
    return lib.or_e5m2(b)


def f16(bits: int) -> float:
    return lib.or_f16(bits)


def e4m3_table() -> np.ndarray:
    return np.array([lib.or_e4m3(b) for b in range(256)], dtype=np.float64)


def to_float32(dtype: str, data: bytes) -> np.ndarray:
    code = {"F32": 0, "BF16": 1, "F16": 2, "F8_E4M3": 3, "F8_E5M2": 4}.get(dtype)
    if code is None:
        raise ValueError(f"Can't decode {dtype} as floats")
    buf = np.frombuffer(bytes(data), dtype=np.uint8).copy()
    out = np.zeros(len(buf), dtype=np.float32)
    n = lib.or_to_float32(code, _ptr(buf), len(buf), _ptr(out))
    return out[:n]


def bf16_bits(x) -> np.ndarray:
    """float32 -> bf16 bits, round to nearest even."""
    return _bf16_bits_np(np.ascontiguousarray(x, dtype=np.float32))


def _bf16_bits_np(x: np.ndarray) -> np.ndarray:
    u = x.view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r.reshape(x.shape)


def bf16_to_f32(bits) -> np.ndarray:
    b = np.ascontiguousarray(bits, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x) -> np.ndarray:
    return bf16_to_f32(_bf16_bits_np(np.ascontiguousarray(x, dtype=np.float32)))


def f32_to_e4m3(v: float) -> int:
    return lib.or_f32_to_e4m3(v)


def f32_to_f16(v: float) -> int:
    return lib.or_f32_to_f16(v)


# ---- noise ----
class MT19937:
    def __init__(self, seed: int):
        self._buf = C.create_string_buffer(624 * 4 + 8)
        lib.or_mt_seed(self._buf, seed)

    def next(self) -> int:
        return lib.or_mt_next(self._buf)


def torch_randn(n: int, seed: int) -> np.ndarray:
    out = np.zeros(n, dtype=np.float32)
    lib.or_torch_randn(n, seed, _ptr(out))
    return out


def lcg(seed: int):
    """The reference tests' LCG (tests/gpu/matmul.test.ts:10-12): returns r() in [0, 1)."""
    state = [seed & 0xFFFFFFFF]

    def r() -> float:
        state[0] = (state[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return state[0] / 2 ** 32

    return r


# ---- matmul ----
def matmul(x, fmt: int, w, m: int, n: int, k: int, scale: float = 1.0, chan_scale=None, gscale=None,
           x_stride=0, w_stride=0, y_stride=0, x_offset=0, w_offset=0, y_offset=0, k_split=1,
           accumulate=False, y=None, y_len=None, threads=None) -> np.ndarray:
    """float64 y = scale * x . W^T (see oracle.h). Returns y (a new float64 array unless given)."""
    x = _c(x, np.float32)
    w = np.ascontiguousarray(w)
    cs = _c(chan_scale, np.float32)
    gs = _c(gscale, np.uint16)
    if y is None:
        ys = y_stride or n
        y = np.zeros(y_len if y_len is not None else y_offset + max(k_split, 1) * m * ys, dtype=np.float64)
    s = MMShape(m, n, k, x_stride, w_stride, y_stride, x_offset, w_offset, y_offset, k_split, int(accumulate))
    if threads is None:
        lib.or_matmul(_ptr(x), fmt, _ptr(w), scale, _ptr(cs), _ptr(gs), C.byref(s), _ptr(y))
    else:
        lib.or_matmul_mt(_ptr(x), fmt, _ptr(w), scale, _ptr(cs), _ptr(gs), C.byref(s), _ptr(y), threads)
    return y


def ksplit_for(m: int, n: int, k: int) -> int:
    return lib.or_ksplit_for(m, n, k)


def rel_error(a, b) -> float:
    a = _c(a, np.float32).ravel()
    b = _c(b, np.float64).ravel()
    return lib.or_rel_error(_ptr(a), _ptr(b), a.size)


def compare(a, b):
    a = _c(a, np.float32).ravel()
    b = _c(b, np.float64).ravel()
    if a.size != b.size:
        raise ValueError(f"Lengths differ: {a.size} vs {b.size}")
    cos, mx, rel = C.c_double(), C.c_double(), C.c_double()
    lib.or_compare(_ptr(a), _ptr(b), a.size, C.byref(cos), C.byref(mx), C.byref(rel))
    return {"cosine": cos.value, "maxError": mx.value, "relativeError": rel.value}


# ---- quantisers ----
def quant_fp8_channel(w, n: int, k: int):
    w = _c(w, np.float32)
    q = np.zeros(n * k, dtype=np.uint8)
    s = np.zeros(n, dtype=np.float32)
    lib.or_quant_fp8_channel(_ptr(w), n, k, _ptr(q), _ptr(s))
    return q, s


def quant_fp8_tensor(w, n: int, k: int):
    w = _c(w, np.float32)
    q = np.zeros(n * k, dtype=np.uint8)
    s = lib.or_quant_fp8_tensor(_ptr(w), n, k, _ptr(q))
    return q, s


def quant_int4_g64(w, n: int, k: int):
    if k % 64:
        raise ValueError("int4 group-64 needs K to be a multiple of 64")
    w = _c(w, np.float32)
    packed = np.zeros(n * k // 2, dtype=np.uint8)
    scales = np.zeros(n * (k // 64), dtype=np.uint16)
    lib.or_quant_int4_g64(_ptr(w), n, k, _ptr(packed), _ptr(scales))
    return packed, scales


def act_split(x_row, terms: int = 2):
    x = _c(x_row, np.float32)
    hi = np.zeros(x.size, dtype=np.uint8)
    lo = np.zeros(x.size, dtype=np.uint8)
    e = C.c_int()
    lib.or_act_split(_ptr(x), x.size, terms, _ptr(hi), _ptr(lo), C.byref(e))
    return hi, lo, e.value


# ---- rmsnorm / rope ----
def rmsnorm(x, w, scale=None, shift=None, eps=1e-5, offset=1.0) -> np.ndarray:
    w = _c(w, np.float32)
    d = w.size
    x = _c(x, np.float32)
    rows = x.size // d
    out = np.zeros(x.size, dtype=np.float64)
    lib.or_rmsnorm(_ptr(x), _ptr(w), _ptr(_c(scale, np.float32)), _ptr(_c(shift, np.float32)), rows, d, eps,
                   offset, _ptr(out))
    return out


def positions(text: int, rows: int, cols: int) -> np.ndarray:
    pos = np.zeros((text + rows * cols) * 3, dtype=np.int64)
    lib.or_positions(text, rows, cols, _ptr(pos))
    return pos.reshape(-1, 3)


def rope_tables(pos, axes=(32, 48, 48), theta=1000.0):
    pos = np.ascontiguousarray(pos, dtype=np.int64)
    tokens, naxes = pos.shape
    ax = np.ascontiguousarray(axes, dtype=np.int64)
    pairs = lib.or_rope_tables(_ptr(pos), tokens, naxes, _ptr(ax), theta, None, None)
    if pairs < 0:
        raise ValueError("Every RoPE axis needs an even number of dims")
    cos = np.zeros(tokens * pairs, dtype=np.float32)
    sin = np.zeros(tokens * pairs, dtype=np.float32)
    lib.or_rope_tables(_ptr(pos), tokens, naxes, _ptr(ax), theta, _ptr(cos), _ptr(sin))
    return cos, sin, pairs


def rope(x, tokens: int, heads: int, pairs: int, cos, sin, pairing: str = "interleaved") -> np.ndarray:
    x = _c(x, np.float32)
    out = np.zeros(x.size, dtype=np.float64)
    lib.or_rope(_ptr(x), tokens, heads, pairs, _ptr(_c(cos, np.float32)), _ptr(_c(sin, np.float32)),
                1 if pairing == "half" else 0, _ptr(out))
    return out


def attention(q, k, v, tokens: int, heads: int, kv_heads: int, dim: int, causal: bool = False) -> np.ndarray:
    """float64 attention of the reference test (tests/gpu/attention.test.ts:9-31)."""
    q, k, v = (_c(a, np.float32) for a in (q, k, v))
    out = np.zeros(tokens * heads * dim, dtype=np.float64)
    lib.or_attention(_ptr(q), _ptr(k), _ptr(v), tokens, heads, kv_heads, dim, int(causal), _ptr(out))
    return out


def block_reference(x, w: dict, cfg: dict, temb, cos, sin) -> np.ndarray:
    """float64 block of the reference test (tests/gpu/block.test.ts:26-100), restated with numpy from the
    formulas: fp8 linears with a scalar or per-channel scale, zero-centred norms (offset 1), GQA attention
    with an optional sigmoid gate, and a SwiGLU or tanh-GELU MLP. w holds host arrays: linears as dicts
    {"bytes", "n", "k", "scale" | "chan_scale"}, norms f32, table f32 [6 hidden]."""
    return joint_block_reference(x, [(0, x.shape[0], w)], cfg, temb, cos, sin)


def _mm(a, lin):
    """a . W^T with W decoded from e4m3 (or given as float), times the scalar or per-channel scale, plus bias."""
    if "bytes" in lin:
        wv = e4m3_table()[lin["bytes"]].reshape(lin["n"], lin["k"])
    else:
        wv = np.asarray(lin["w"], np.float64).reshape(lin["n"], lin["k"])
    y = np.asarray(a, np.float64).reshape(-1, lin["k"]) @ wv.T
    y = y * (lin["chan_scale"].astype(np.float64) if lin.get("chan_scale") is not None else lin.get("scale", 1.0))
    if lin.get("bias") is not None:
        y = y + lin["bias"].astype(np.float64)
    return y


def _rms(a, wt, rows, d, sc=None, sh=None, eps=1e-5, offset=1.0):
    """RMSNorm with modulation (src/kernels/rmsnorm.ts:42-46) in float64."""
    a = np.asarray(a, np.float64).reshape(rows, d)
    inv = 1.0 / np.sqrt((a * a).sum(1) / d + eps)
    y = a * inv[:, None] * (offset + np.asarray(wt, np.float64))
    if sc is not None:
        y = y * (1.0 + sc) + sh
    return y


def _gelu(u):
    return 0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))


def block_rows_reference(x, w: dict, cfg: dict, temb, cos, sin, rows) -> np.ndarray:
    """The float64 single-stream block's output on the given rows only: keys and values come from every token, the
    queries and everything after attention from `rows` alone (the same formulas as joint_block_reference, for
    checking a few rows of a full-size block without the full block's float64 cost)."""
    return joint_block_reference(x, [(0, x.shape[0], w)], cfg, temb, cos, sin, rows=rows)


def joint_block_reference(x, parts: list, cfg: dict, temb, cos, sin, rows=None) -> np.ndarray:
    """float64 block over a token sequence split into parts (row0, rows, w): each part has its own weights and
    modulation, attention runs over all rows. One part = the single-stream block of tests/gpu/block.test.ts:26-100;
    two parts (text rows, image rows) = the double-stream block built from the same ops. rows: a list of row
    indices (one part only) to return the output of just those rows, in that order."""
    if rows is not None:
        return _block_rows(np.asarray(x, np.float64), parts, cfg, temb, cos, sin, np.asarray(rows))
    t, hid, heads, kvh, hd = x.shape[0], cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    eps = cfg.get("eps", 1e-5)
    pairs = hd // 2

    def rope_np(a, r0, tokens, nh):
        a = a.reshape(tokens, nh, pairs, 2)
        c = cos.reshape(-1, pairs)[r0:r0 + tokens].reshape(tokens, 1, pairs).astype(np.float64)
        s = sin.reshape(-1, pairs)[r0:r0 + tokens].reshape(tokens, 1, pairs).astype(np.float64)
        out = np.empty_like(a)
        out[..., 0] = a[..., 0] * c - a[..., 1] * s
        out[..., 1] = a[..., 1] * c + a[..., 0] * s
        return out.reshape(tokens, nh * hd)

    x = np.asarray(x, np.float64)
    q, k, v = np.empty((t, heads, hd)), np.empty((t, kvh, hd)), np.empty((t, kvh, hd))
    hs, mods = [], []
    for r0, n, w in parts:
        mod = [(np.asarray(temb[i * hid:(i + 1) * hid], np.float64) + w["table"][i * hid:(i + 1) * hid])
               for i in range(6)]
        h = _rms(x[r0:r0 + n], w["norm1"], n, hid, mod[0], mod[1], eps)
        q[r0:r0 + n] = rope_np(_rms(_mm(h, w["wq"]), w["norm_q"], n * heads, hd, eps=eps), r0, n, heads).reshape(n, heads, hd)
        k[r0:r0 + n] = rope_np(_rms(_mm(h, w["wk"]), w["norm_k"], n * kvh, hd, eps=eps), r0, n, kvh).reshape(n, kvh, hd)
        v[r0:r0 + n] = _mm(h, w["wv"]).reshape(n, kvh, hd)
        hs.append(h)
        mods.append(mod)
    o = np.empty((t, heads, hd))
    for hh in range(heads):
        g = hh // (heads // kvh)
        s = q[:, hh] @ k[:, g].T / np.sqrt(hd)
        p = np.exp(s - s.max(1, keepdims=True))
        o[:, hh] = (p / p.sum(1, keepdims=True)) @ v[:, g]
    o = o.reshape(t, hid)
    out = np.empty_like(x)
    for (r0, n, w), h, mod in zip(parts, hs, mods):
        prescale, preshift, pregate, postscale, postshift, postgate = mod
        op = o[r0:r0 + n]
        if cfg.get("attn_gate", True):
            op = op / (1.0 + np.exp(-_mm(h, w["gate"])))
        x1 = x[r0:r0 + n] + pregate * _mm(op, w["wo"])
        h2 = _rms(x1, w["norm2"], n, hid, postscale, postshift, eps)
        if cfg.get("mlp_act", "swiglu") == "swiglu":
            gg = _mm(h2, w["mlp_gate"])
            m = gg / (1.0 + np.exp(-gg)) * _mm(h2, w["mlp_up"])
        else:
            m = _gelu(_mm(h2, w["mlp_up"]))
        out[r0:r0 + n] = x1 + postgate * _mm(m, w["mlp_down"])
    return out


def _block_rows(x, parts, cfg, temb, cos, sin, rows):
    """joint_block_reference restricted to output rows `rows` of a one-part block."""
    if len(parts) != 1:
        raise ValueError("row sampling takes a one-part block")
    (_, t, w), = parts
    hid, heads, kvh, hd = cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    eps, pairs = cfg.get("eps", 1e-5), hd // 2
    mod = [(np.asarray(temb[i * hid:(i + 1) * hid], np.float64) + w["table"][i * hid:(i + 1) * hid]) for i in range(6)]
    prescale, preshift, pregate, postscale, postshift, postgate = mod
    cs, sn = (np.asarray(a, np.float64).reshape(-1, pairs) for a in (cos, sin))

    def rope_np(a, idx, nh):
        a = a.reshape(len(idx), nh, pairs, 2)
        c, s = cs[idx][:, None, :], sn[idx][:, None, :]
        out = np.empty_like(a)
        out[..., 0] = a[..., 0] * c - a[..., 1] * s
        out[..., 1] = a[..., 1] * c + a[..., 0] * s
        return out.reshape(len(idx), nh, hd)

    allr = np.arange(t)
    h = _rms(x, w["norm1"], t, hid, prescale, preshift, eps)
    k = rope_np(_rms(_mm(h, w["wk"]), w["norm_k"], t * kvh, hd, eps=eps), allr, kvh)
    v = _mm(h, w["wv"]).reshape(t, kvh, hd)
    hr = h[rows]
    q = rope_np(_rms(_mm(hr, w["wq"]), w["norm_q"], len(rows) * heads, hd, eps=eps), rows, heads)
    o = np.empty((len(rows), heads, hd))
    for hh in range(heads):
        g = hh // (heads // kvh)
        s = q[:, hh] @ k[:, g].T / np.sqrt(hd)
        p = np.exp(s - s.max(1, keepdims=True))
        o[:, hh] = (p / p.sum(1, keepdims=True)) @ v[:, g]
    op = o.reshape(len(rows), hid)
    if cfg.get("attn_gate", True):
        op = op / (1.0 + np.exp(-_mm(hr, w["gate"])))
    x1 = x[rows] + pregate * _mm(op, w["wo"])
    h2 = _rms(x1, w["norm2"], len(rows), hid, postscale, postshift, eps)
    if cfg.get("mlp_act", "swiglu") == "swiglu":
        gg = _mm(h2, w["mlp_gate"])
        m = gg / (1.0 + np.exp(-gg)) * _mm(h2, w["mlp_up"])
    else:
        m = _gelu(_mm(h2, w["mlp_up"]))
    return x1 + postgate * _mm(m, w["mlp_down"])


# ---------------- the step driver's host parts (src/model/transformer.ts, src/model/sampler.ts) ----------------
def timestep_embedding(timestep: float, dim: int = 256) -> np.ndarray:
    """[cos(1000 t f_i), sin(1000 t f_i)], f_i = 10000^(-i / (dim/2)), cos first (transformer.ts:41-51)."""
    half = dim // 2
    arg = 1000.0 * timestep * np.exp(-np.log(10000.0) * np.arange(half) / half)
    return np.concatenate([np.cos(arg), np.sin(arg)]).astype(np.float32)


def patch_grid(height: int, width: int):
    return (height + 1) // 2, (width + 1) // 2


def patchify(latent, height: int, width: int, channels: int = 16) -> np.ndarray:
    """Latent [C, H, W] -> tokens [rows*cols, 4C], feature (channel, patch row, patch col); odd sizes wrap
    (transformer.ts:59-69). A loop restatement of the reference's index formula."""
    lat = np.asarray(latent).reshape(channels, height, width)
    rows, cols = patch_grid(height, width)
    out = np.empty((rows * cols, channels * 4), dtype=lat.dtype)
    for r in range(rows):
        for c in range(cols):
            for pr in range(2):
                for pc in range(2):
                    out[r * cols + c, np.arange(channels) * 4 + pr * 2 + pc] = \
                        lat[:, (r * 2 + pr) % height, (c * 2 + pc) % width]
    return out.reshape(-1)


def unpatchify(tokens, height: int, width: int, channels: int = 16) -> np.ndarray:
    """The inverse of patchify; the padding is cropped off (transformer.ts:72-82)."""
    rows, cols = patch_grid(height, width)
    tok = np.asarray(tokens).reshape(rows * cols, channels * 4)
    out = np.empty((channels, height, width), dtype=tok.dtype)
    for y in range(height):
        for x in range(width):
            out[:, y, x] = tok[(y // 2) * cols + x // 2, np.arange(channels) * 4 + (y % 2) * 2 + (x % 2)]
    return out.reshape(-1)


def sigmas(steps: int = 8, mu: float = 1.15) -> list:
    """linspace(1, 1/steps, steps) under the exponential time shift, then 0 (src/model/sampler.ts:9-19)."""
    raw = [1 - i * (1 - 1 / steps) / ((steps - 1) or 1) for i in range(steps)]
    return [float(np.exp(mu) / (np.exp(mu) + (1 / s - 1))) for s in raw] + [0.0]


def euler_step(x, velocity, sigma: float, nxt: float) -> np.ndarray:
    """x + (sigma_next - sigma) v, in f32 like the reference's Float32Array (sampler.ts:22-24)."""
    return (np.asarray(x, np.float32) + np.float32(nxt - sigma) * np.asarray(velocity, np.float32)).astype(np.float32)


def gaussian(n: int, seed: int) -> np.ndarray:
    """Seeded Box-Muller normals from a 32-bit LCG (sampler.ts:27-38): u = (s + 0.5) / 2^32 per draw."""
    s = (seed & 0xFFFFFFFF) or 1
    out = np.empty(n, dtype=np.float32)
    for i in range(0, n, 2):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        u1 = (s + 0.5) / 2 ** 32
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        u2 = (s + 0.5) / 2 ** 32
        r, a = np.sqrt(-2 * np.log(u1)), 2 * np.pi * u2
        out[i] = r * np.cos(a)
        if i + 1 < n:
            out[i + 1] = r * np.sin(a)
    return out


def step_reference(latent, height: int, width: int, timestep: float, ctx, w: dict, cfg: dict) -> np.ndarray:
    """float64 denoising step (transformer.ts:134-176) of a Flux-style layout: time MLP, text projection,
    patchify + first linear, `double` two-part blocks over [text, image] rows, `single` one-part blocks, the
    modulated last norm and linear, unpatchify. w: {"first", "tmlp0", "tmlp2", "tproj", "txt_in", "last_linear":
    linear dicts; "double": [(txt, img)], "single": [block dicts]; "last_norm", "last_scale", "last_shift"}."""
    hid, ch = cfg["hidden"], cfg.get("channels", 16)
    rows, cols = patch_grid(height, width)
    ctx = np.asarray(ctx, np.float64).reshape(-1, w["txt_in"]["k"])
    L = ctx.shape[0]
    T = L + rows * cols
    emb = timestep_embedding(timestep, cfg.get("time_dim", 256)).astype(np.float64)
    t = _mm(_gelu(_mm(emb, w["tmlp0"])), w["tmlp2"]).reshape(-1)
    tvec = _mm(_gelu(t), w["tproj"]).reshape(-1)
    img = _mm(patchify(np.asarray(latent, np.float32), height, width, ch), w["first"])
    x = np.concatenate([_mm(ctx, w["txt_in"]), img])
    cos, sin, pairs = rope_tables(positions(L, rows, cols), cfg["axes"], cfg["theta"])
    for txt_w, img_w in w["double"]:
        x = joint_block_reference(x, [(0, L, txt_w), (L, T - L, img_w)], cfg, tvec, cos, sin)
    for bw in w["single"]:
        x = joint_block_reference(x, [(0, T, bw)], cfg, tvec, cos, sin)
    scale = t + w["last_scale"].astype(np.float64)
    shift = t + w["last_shift"].astype(np.float64)
    last = _mm(_rms(x, w["last_norm"], T, hid, scale, shift, cfg.get("eps", 1e-5)), w["last_linear"])
    return unpatchify(last[L:], height, width, ch)
