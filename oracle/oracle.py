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
    t, hid, heads, kvh, hd = x.shape[0], cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["head_dim"]
    eps = cfg.get("eps", 1e-5)
    e4 = e4m3_table()

    def mm(a, lin):
        wv = e4[lin["bytes"]].reshape(lin["n"], lin["k"])
        y = a @ wv.T
        return y * (lin["chan_scale"].astype(np.float64) if lin.get("chan_scale") is not None else lin["scale"])

    def rms(a, wt, rows, d, sc=None, sh=None):
        a = a.reshape(rows, d)
        inv = 1.0 / np.sqrt((a * a).sum(1) / d + eps)
        y = a * inv[:, None] * (1.0 + wt.astype(np.float64))
        if sc is not None:
            y = y * (1.0 + sc) + sh
        return y

    def rope_np(a, tokens, nh):
        pairs = hd // 2
        a = a.reshape(tokens, nh, pairs, 2)
        c = cos.reshape(tokens, 1, pairs).astype(np.float64)
        s = sin.reshape(tokens, 1, pairs).astype(np.float64)
        out = np.empty_like(a)
        out[..., 0] = a[..., 0] * c - a[..., 1] * s
        out[..., 1] = a[..., 1] * c + a[..., 0] * s
        return out.reshape(tokens, nh * hd)

    x = x.astype(np.float64)
    mod = [(temb[i * hid:(i + 1) * hid].astype(np.float64) + w["table"][i * hid:(i + 1) * hid]) for i in range(6)]
    prescale, preshift, pregate, postscale, postshift, postgate = mod
    h = rms(x, w["norm1"], t, hid, prescale, preshift)
    q = rope_np(rms(mm(h, w["wq"]), w["norm_q"], t * heads, hd), t, heads).reshape(t, heads, hd)
    k = rope_np(rms(mm(h, w["wk"]), w["norm_k"], t * kvh, hd), t, kvh).reshape(t, kvh, hd)
    v = mm(h, w["wv"]).reshape(t, kvh, hd)
    o = np.empty((t, heads, hd))
    for hh in range(heads):
        g = hh // (heads // kvh)
        s = q[:, hh] @ k[:, g].T / np.sqrt(hd)
        p = np.exp(s - s.max(1, keepdims=True))
        o[:, hh] = (p / p.sum(1, keepdims=True)) @ v[:, g]
    o = o.reshape(t, hid)
    if cfg.get("attn_gate", True):
        o = o / (1.0 + np.exp(-mm(h, w["gate"])))
    x1 = x + pregate * mm(o, w["wo"])
    h2 = rms(x1, w["norm2"], t, hid, postscale, postshift)
    if cfg.get("mlp_act", "swiglu") == "swiglu":
        gg = mm(h2, w["mlp_gate"])
        m = gg / (1.0 + np.exp(-gg)) * mm(h2, w["mlp_up"])
    else:
        u = mm(h2, w["mlp_up"])
        m = 0.5 * u * (1.0 + np.tanh(0.7978845608028654 * (u + 0.044715 * u ** 3)))
    return x1 + postgate * mm(m, w["mlp_down"])
