"""The operator API of the hot path, mirroring src/model/ops.ts.

Each op takes device buffers, queues its kernel(s) on the Graph's stream through the C ABI and
returns a new pooled output buffer, like the reference's graph steps:

    linear(graph, x, w, m)                          ops.ts:61-73
    norm(graph, x, weight, rows, d, mod, eps, offset)  ops.ts:78-82
    no_mod(graph, d)                                ops.ts:85
    rotate(graph, x, heads, rope, pairing)          ops.ts:89-93
    k_split_for(m, n, k)                            ops.ts:42-45

The reference's buffers hold f32; here each op also names the element type of its activations
(``x_dtype`` / ``y_dtype`` / ``out_dtype``: "f32" or "bf16"), f32 by default.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional

from . import _lib as L
from .graph import Buffer, Graph, addr


@dataclass
class Linear:
    """A linear layer (ops.ts:24-32): W [n, k] as stored.

    dtype: "fp8" (e4m3 bytes) | "bf16" | "f32" | "int4" (group-64, needs group_scale f16 [n, k/64]).
    scale: the scalar weight_scale; chan_scale: optional per-output-channel f32 [n] (replaces scale).
    lora: optional (down [rank, k], up [n, rank]) with up.scale = strength * alpha / rank.
    """

    buffer: object
    dtype: str
    scale: float
    n: int
    k: int
    bias: object = None
    lora: Optional[tuple] = None
    chan_scale: object = None
    group_scale: object = None

    def desc(self, keep: list) -> L.LinearDesc:
        d = L.LinearDesc(addr(self.buffer).value, L.DTYPES[self.dtype], self.scale, addr(self.chan_scale).value,
                         addr(self.group_scale).value, self.n, self.k, addr(self.bias).value, None, None)
        if self.lora is not None:
            down, up = self.lora
            dd, du = down.desc(keep), up.desc(keep)
            keep.extend([dd, du])
            d.lora_down = C.pointer(dd)
            d.lora_up = C.pointer(du)
        return d


def k_split_for(m: int, n: int, k: int) -> int:
    """How many K slices make x[m, k] . W^T (n narrow) fill the GPU: 1 = no split (ops.ts:42-45)."""
    return L.lib().we_ksplit_for(m, n, k)


def linear(graph: Graph, x, w: Linear, m: int, x_dtype: str = "f32", y_dtype: str = "f32",
           fast: bool = False) -> Buffer:
    """y[m, n] = x[m, k] . W^T (+ bias) (+ up.scale (x . down^T) . up^T) (ops.ts:61-73).

    bf16 x with fp8 W runs on tcgen05 (two e4m3 activation terms: exact for bf16 x); fast=True
    uses one term (fp8 tensor peak, ~3% rms activation rounding)."""
    keep: list = []
    d = w.desc(keep)
    out = C.c_void_p()
    flags = L.MM_FP8_FAST if fast else 0
    L.check(graph.ctx, L.lib().we_linear_forward(graph.ctx, addr(x), L.DTYPES[x_dtype], C.byref(d), m,
                                                 L.DTYPES[y_dtype], flags, C.byref(out)))
    return Buffer(out.value, m * w.n * L.DTYPE_BYTES[L.DTYPES[y_dtype]])


def linear_host(graph: Graph, x_host, w: Linear, m: int, y_host, x_dtype: str = "bf16", y_dtype: str = "bf16",
                fast: bool = False, chunk_rows: int = 0) -> None:
    """y_host[m, n] = linear(x_host[m, k]) from host memory to host memory in one call: the upload, the linear
    (ops.ts:61-73) and the read-back (graph.ts:108-119), row chunk by row chunk on three streams so that both
    copies overlap the GEMMs. x_host / y_host are CPU tensors (page-locked for the overlap) or host addresses.
    Returns when y_host holds the result."""
    keep: list = []
    d = w.desc(keep)
    flags = L.MM_FP8_FAST if fast else 0
    L.check(graph.ctx, L.lib().we_linear_host(graph.ctx, addr(x_host), L.DTYPES[x_dtype], C.byref(d), m,
                                              L.DTYPES[y_dtype], flags, addr(y_host), chunk_rows))


@dataclass
class Mod:
    """Modulation vectors of length d (ops.ts:75); None = zeros."""

    scale: object = None
    shift: object = None


def no_mod(graph: Graph, d: int) -> Mod:
    """Zero scale and shift of length d (ops.ts:85)."""
    m = L.ModDesc()
    L.check(graph.ctx, L.lib().we_no_mod(graph.ctx, d, C.byref(m)))
    return Mod(Buffer(m.scale, d * 4), Buffer(m.shift, d * 4))


def norm(graph: Graph, x, weight, rows: int, d: int, mod: Mod | None = None, eps: float = 1e-5,
         offset: float = 1.0, x_dtype: str = "f32", out_dtype: str = "f32") -> Buffer:
    """RMSNorm per row of length d, then (1 + scale) . + shift (ops.ts:78-82). offset 1: zero-centred
    weight (Krea 2), 0: plain."""
    mod = mod or Mod()
    md = L.ModDesc(addr(mod.scale).value, addr(mod.shift).value)
    out = C.c_void_p()
    L.check(graph.ctx, L.lib().we_norm(graph.ctx, addr(x), L.DTYPES[x_dtype], addr(weight), rows, d, C.byref(md), eps,
                                       offset, L.DTYPES[out_dtype], C.byref(out)))
    return Buffer(out.value, rows * d * L.DTYPE_BYTES[L.DTYPES[out_dtype]])


@dataclass
class Rope:
    """cos/sin tables [tokens, pairs] on the device (ops.ts:87)."""

    cos: object
    sin: object
    pairs: int
    tokens: int


def rotate(graph: Graph, x, heads: int, rope: Rope, pairing: str = "interleaved", x_dtype: str = "f32",
           out_dtype: str = "f32") -> Buffer:
    """RoPE over x [tokens, heads, 2 pairs] (ops.ts:89-93)."""
    rd = L.RopeDesc(addr(rope.cos).value, addr(rope.sin).value, rope.pairs, rope.tokens)
    out = C.c_void_p()
    p = L.ROPE_HALF if pairing == "half" else L.ROPE_INTERLEAVED
    L.check(graph.ctx, L.lib().we_rotate(graph.ctx, addr(x), L.DTYPES[x_dtype], heads, C.byref(rd), p,
                                         L.DTYPES[out_dtype], C.byref(out)))
    return Buffer(out.value, rope.tokens * heads * rope.pairs * 2 * L.DTYPE_BYTES[L.DTYPES[out_dtype]])


def qk_norm_rotate(graph: Graph, x, weight, heads: int, rope: Rope, eps: float = 1e-5, offset: float = 1.0,
                   pairing: str = "interleaved", x_dtype: str = "f32", out_dtype: str = "f32") -> Buffer:
    """norm(x, weight, tokens*heads, head_dim) then rotate, in one pass (src/model/block.ts:53-56)."""
    nbytes = rope.tokens * heads * rope.pairs * 2 * L.DTYPE_BYTES[L.DTYPES[out_dtype]]
    out = graph.buffer(nbytes)
    p = L.ROPE_HALF if pairing == "half" else L.ROPE_INTERLEAVED
    L.check(graph.ctx, L.lib().we_qknorm_rope(graph.ctx, addr(x), L.DTYPES[x_dtype], addr(weight), eps, offset,
                                              addr(rope.cos), addr(rope.sin), rope.tokens, heads, rope.pairs, p,
                                              addr(out), L.DTYPES[out_dtype]))
    return out


def attention(graph: Graph, q, k, v, tokens: int, heads: int, kv_heads: int, dim: int, causal: bool = False,
              chunk: int | None = None, dtype: str = "f32", out_dtype: str | None = None) -> Buffer:
    """attention(graph, q, k, v, shape) (src/kernels/attention.ts:20-51): softmax(q k^T / sqrt(dim)) v with
    grouped-query heads; q [tokens, heads, dim], k, v [tokens, kv_heads, dim] -> a new [tokens, heads, dim].
    `chunk` only bounded the reference's score memory; the kernels here keep no score matrix."""
    od = out_dtype or dtype
    out = C.c_void_p()
    L.check(graph.ctx, L.lib().we_attend(graph.ctx, addr(q), addr(k), addr(v), L.DTYPES[dtype], tokens, heads,
                                         kv_heads, dim, int(causal), L.DTYPES[od], C.byref(out)))
    return Buffer(out.value, tokens * heads * dim * L.DTYPE_BYTES[L.DTYPES[od]])


def elementwise(graph: Graph, op: str, a, b, n: int, g=None, d: int = 1, dtype: str = "f32",
                out_dtype: str | None = None) -> Buffer:
    """One per-value step as a graph op (ops.ts:95-99): a new buffer of n values."""
    od = out_dtype or dtype
    out = C.c_void_p()
    L.check(graph.ctx, L.lib().we_ew(graph.ctx, L.EW[op], addr(a), addr(b), addr(g), n, d, L.DTYPES[dtype],
                                     L.DTYPES[od], C.byref(out)))
    return Buffer(out.value, n * L.DTYPE_BYTES[L.DTYPES[od]])


def swiglu(graph: Graph, gate, up, n: int, dtype: str = "f32") -> Buffer:
    """silu(gate) . up (ops.ts:102)"""
    return elementwise(graph, "swiglu", gate, up, n, dtype=dtype)


def sigmoid_gate(graph: Graph, a, gate, n: int, dtype: str = "f32") -> Buffer:
    """a . sigmoid(gate) (ops.ts:104)"""
    return elementwise(graph, "sigmoid_gate", a, gate, n, dtype=dtype)


def gated_add(graph: Graph, x, h, g, n: int, d: int, dtype: str = "f32") -> Buffer:
    """x + g[column] . h, g of length d (ops.ts:106-107)"""
    return elementwise(graph, "gated_add", x, h, n, g=g, d=d, dtype=dtype)


def add(graph: Graph, x, h, n: int, dtype: str = "f32") -> Buffer:
    """x + h (ops.ts:109)"""
    return elementwise(graph, "add", x, h, n, dtype=dtype)


def gelu(graph: Graph, x, n: int, dtype: str = "f32") -> Buffer:
    """GELU, tanh form (ops.ts:111)"""
    return elementwise(graph, "gelu_tanh", x, None, n, dtype=dtype)


def silu(graph: Graph, x, n: int, dtype: str = "f32") -> Buffer:
    """x . sigmoid(x) (ops.ts:113)"""
    return elementwise(graph, "silu", x, None, n, dtype=dtype)
