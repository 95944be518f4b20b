"""Kernel-level entry points, mirroring src/kernels/{matmul,fp8,rmsnorm,rope}.ts.

``matmul`` is matmulWgsl + matmulParams on device buffers; ``matmul_fp8`` / ``matmul_bf16`` /
``matmul_f32`` / ``unpack_fp8`` / ``rmsnorm_once`` / ``rope_once`` are the reference's one-shot
runners (upload, run once, read back) that its GPU tests call. ``rope_tables`` and ``positions``
are the host-side table builders (float64, like src/kernels/rope.ts:14-36).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib as L
from .graph import Buffer, Graph, addr

AXES = (32, 48, 48)  # src/kernels/rope.ts:10 (Krea 2)
THETA = 1000.0       # src/kernels/rope.ts:11
TILE = 128           # src/kernels/matmul.ts:33


def matmul_params(m: int, n: int, k: int, scale: float, x_stride=None, w_stride=None, y_stride=None, x_offset=0,
                  w_offset=0, y_offset=0, k_split=1) -> L.MatmulDesc:
    """matmulParams (src/kernels/matmul.ts:198-212): validates like the reference and returns the descriptor."""
    xs = k if x_stride is None else x_stride
    ws = k if w_stride is None else w_stride
    ys = n if y_stride is None else y_stride
    for name, v in (("K", k), ("xStride", xs), ("wStride", ws), ("xOffset", x_offset), ("wOffset", w_offset)):
        if v % 4:
            raise ValueError(f"{name} must be a multiple of 4, got {v}")
    return L.MatmulDesc(m, n, k, xs, ws, ys, x_offset, w_offset, y_offset, k_split, scale, None, None, None,
                        L.F32, L.FP8, L.F32, 0)


def epilogue(act=None, aux_op=None, aux=None, aux_dtype="f32", gate=None) -> L.Epilogue:
    """Fused per-value steps after a matmul (see we_epilogue): act "gelu_tanh" | "silu"; aux_op
    "sigmoid_gate" (aux * sigmoid(v)) | "swiglu" (silu(aux) * v); gate: per-column factor [n]."""
    return L.Epilogue(L.ACTS[act], L.AUX_OPS[aux_op], L.DTYPES[aux_dtype], addr(aux).value, addr(gate).value)


def matmul(graph: Graph, x, w, y, m: int, n: int, k: int, scale: float = 1.0, *, x_dtype="f32", w_dtype="fp8",
           y_dtype="f32", chan_scale=None, group_scale=None, bias=None, x_stride=None, w_stride=None, y_stride=None,
           x_offset=0, w_offset=0, y_offset=0, k_split=1, accumulate=False, fast=False, force_simt=False,
           act=None, aux_op=None, aux=None, aux_dtype="f32", gate=None) -> None:
    """Queues y = x . W^T * scale (matmulWgsl, src/kernels/matmul.ts:118-178) on device buffers, with optional
    fused epilogue steps (act, aux_op/aux, gate; see `epilogue`)."""
    d = matmul_params(m, n, k, scale, x_stride, w_stride, y_stride, x_offset, w_offset, y_offset, k_split)
    d.epi = epilogue(act, aux_op, aux, aux_dtype, gate)
    d.chan_scale = addr(chan_scale).value
    d.group_scale = addr(group_scale).value
    d.bias = addr(bias).value
    d.x_dtype, d.w_dtype, d.y_dtype = L.DTYPES[x_dtype], L.DTYPES[w_dtype], L.DTYPES[y_dtype]
    d.flags = (L.MM_ACCUMULATE if accumulate else 0) | (L.MM_FP8_FAST if fast else 0) | (
        L.MM_FORCE_SIMT if force_simt else 0)
    L.check(graph.ctx, L.lib().we_matmul(graph.ctx, C.byref(d), addr(x), addr(w), addr(y)))


def matmul_workgroups(m: int, n: int) -> tuple:
    """matmulWorkgroups (src/kernels/matmul.ts:214): 128 x 128 tiles of the reference shader."""
    return (-(-n // TILE), -(-m // TILE))


def _pad4(b: np.ndarray) -> np.ndarray:
    out = np.zeros(-(-b.nbytes // 4) * 4, np.uint8)
    out[: b.nbytes] = b.view(np.uint8).ravel()
    return out


def matmul_fp8(graph: Graph, x: np.ndarray, w: np.ndarray, scale: float, m: int, n: int, k: int, **kw) -> np.ndarray:
    """One-shot fp8 run (matmulFp8, src/kernels/matmul.ts:223-235): f32 x [m, k], e4m3 bytes w [n, k]."""
    if x.size != m * k or w.size != n * k:
        raise ValueError("x or w does not match the shape")
    mark = graph.mark()
    try:
        xb, wb, yb = graph.buffer(np.asarray(x, np.float32)), graph.buffer(_pad4(np.asarray(w, np.uint8))), graph.buffer(m * n * 4)
        matmul(graph, xb, wb, yb, m, n, k, scale, w_dtype="fp8", **kw)
        return graph.read(yb, m * n * 4, np.float32).copy()
    finally:
        graph.release(mark)


def matmul_bf16(graph: Graph, x: np.ndarray, w: np.ndarray, scale: float, m: int, n: int, k: int, **kw) -> np.ndarray:
    """One-shot run with bf16 W [n, k] given as little-endian bytes (matmulBf16, matmul.ts:238-248)."""
    if x.size != m * k or w.nbytes != n * k * 2:
        raise ValueError("x or w does not match the shape")
    mark = graph.mark()
    try:
        xb, wb, yb = graph.buffer(np.asarray(x, np.float32)), graph.buffer(_pad4(np.asarray(w))), graph.buffer(m * n * 4)
        matmul(graph, xb, wb, yb, m, n, k, scale, w_dtype="bf16", **kw)
        return graph.read(yb, m * n * 4, np.float32).copy()
    finally:
        graph.release(mark)


def matmul_f32(graph: Graph, x: np.ndarray, w: np.ndarray, scale: float, m: int, n: int, k: int,
               output_length: int | None = None, **layout) -> np.ndarray:
    """One-shot f32 run with any layout; output_length is the size of y in values (matmul.ts:251-265)."""
    out_len = m * n if output_length is None else output_length
    mark = graph.mark()
    try:
        xb, wb, yb = graph.buffer(np.asarray(x, np.float32)), graph.buffer(np.asarray(w, np.float32)), graph.buffer(out_len * 4)
        matmul(graph, xb, wb, yb, m, n, k, scale, w_dtype="f32", **layout)
        return graph.read(yb, out_len * 4, np.float32).copy()
    finally:
        graph.release(mark)


def unpack_fp8(graph: Graph, data: np.ndarray, scale: float) -> np.ndarray:
    """unpackFp8 (src/kernels/fp8.ts:24-36): out[i] = e4m3(bytes[i]) * scale."""
    n = data.size
    mark = graph.mark()
    try:
        ib, ob = graph.buffer(_pad4(np.asarray(data, np.uint8))), graph.buffer(n * 4)
        L.check(graph.ctx, L.lib().we_unpack_fp8(graph.ctx, addr(ib), n, scale, addr(ob)))
        return graph.read(ob, n * 4, np.float32).copy()
    finally:
        graph.release(mark)


def rmsnorm(graph: Graph, x, weight, rows: int, d: int, out, scale=None, shift=None, eps: float = 1e-5,
            offset: float = 1.0, x_dtype="f32", out_dtype="f32") -> None:
    """rmsnormWgsl on device buffers (src/kernels/rmsnorm.ts:13-48)."""
    L.check(graph.ctx, L.lib().we_rmsnorm(graph.ctx, addr(x), L.DTYPES[x_dtype], addr(weight), addr(scale),
                                          addr(shift), rows, d, eps, offset, addr(out), L.DTYPES[out_dtype]))


def rmsnorm_once(graph: Graph, x: np.ndarray, weight: np.ndarray, eps: float = 1e-5, offset: float = 1.0,
                 scale=None, shift=None) -> np.ndarray:
    """One-shot run (rmsnorm, src/kernels/rmsnorm.ts:62-74)."""
    d = weight.size
    if x.size % d:
        raise ValueError("x is not a whole number of rows")
    rows = x.size // d
    mark = graph.mark()
    try:
        xb, wb, ob = graph.buffer(np.asarray(x, np.float32)), graph.buffer(np.asarray(weight, np.float32)), graph.buffer(x.size * 4)
        sc = graph.buffer(np.asarray(scale, np.float32)) if scale is not None else None
        sh = graph.buffer(np.asarray(shift, np.float32)) if shift is not None else None
        rmsnorm(graph, xb, wb, rows, d, ob, sc, sh, eps, offset)
        return graph.read(ob, x.size * 4, np.float32).copy()
    finally:
        graph.release(mark)


def rope_tables(pos, axes=AXES, theta: float = THETA):
    """ropeTables (src/kernels/rope.ts:20-36): cos/sin [tokens, pairs] f32 from float64 angles."""
    p = np.ascontiguousarray(pos, dtype=np.int64)
    if p.ndim == 1:
        p = p[:, None]
    ax = np.ascontiguousarray(axes, dtype=np.int64)
    pairs = L.lib().we_rope_tables(p.ctypes.data_as(C.c_void_p), p.shape[0], ax.size, ax.ctypes.data_as(C.c_void_p),
                                   theta, None, None)
    if pairs < 0:
        raise ValueError("Every RoPE axis needs an even number of dims")
    cos = np.zeros(p.shape[0] * pairs, np.float32)
    sin = np.zeros(p.shape[0] * pairs, np.float32)
    L.lib().we_rope_tables(p.ctypes.data_as(C.c_void_p), p.shape[0], ax.size, ax.ctypes.data_as(C.c_void_p), theta,
                           cos.ctypes.data_as(C.c_void_p), sin.ctypes.data_as(C.c_void_p))
    return cos, sin, int(pairs)


def positions(text: int, rows: int, cols: int) -> np.ndarray:
    """positions (src/kernels/rope.ts:14-18): text at (0,0,0), then image tokens (0, row, col)."""
    pos = np.zeros((text + rows * cols, 3), np.int64)
    if L.lib().we_positions(text, rows, cols, pos.ctypes.data_as(C.c_void_p)) != L.WE_OK:
        raise ValueError("negative size")
    return pos


def rope_apply(graph: Graph, x, cos, sin, tokens: int, heads: int, pairs: int, out, pairing="interleaved",
               x_dtype="f32", out_dtype="f32") -> None:
    """ropeKernel on device buffers (src/kernels/rope.ts:59-77)."""
    p = L.ROPE_HALF if pairing == "half" else L.ROPE_INTERLEAVED
    L.check(graph.ctx, L.lib().we_rope_apply(graph.ctx, addr(x), L.DTYPES[x_dtype], addr(cos), addr(sin), tokens,
                                             heads, pairs, p, addr(out), L.DTYPES[out_dtype]))


def rope_once(graph: Graph, x: np.ndarray, heads: int, tables, pairing: str = "interleaved") -> np.ndarray:
    """One-shot run (rope, src/kernels/rope.ts:89-99)."""
    cos, sin, pairs = tables
    tokens = cos.size // pairs
    if x.size != tokens * heads * pairs * 2:
        raise ValueError("x does not match tokens × heads × head dim")
    mark = graph.mark()
    try:
        xb, cb, sb, ob = (graph.buffer(np.asarray(x, np.float32)), graph.buffer(cos), graph.buffer(sin),
                          graph.buffer(x.size * 4))
        rope_apply(graph, xb, cb, sb, tokens, heads, pairs, ob, pairing)
        return graph.read(ob, x.size * 4, np.float32).copy()
    finally:
        graph.release(mark)


def qknorm_rope(graph: Graph, x, weight, cos, sin, tokens: int, heads: int, pairs: int, out, eps=1e-5, offset=1.0,
                pairing="interleaved", x_dtype="f32", out_dtype="f32") -> None:
    p = L.ROPE_HALF if pairing == "half" else L.ROPE_INTERLEAVED
    L.check(graph.ctx, L.lib().we_qknorm_rope(graph.ctx, addr(x), L.DTYPES[x_dtype], addr(weight), eps, offset,
                                              addr(cos), addr(sin), tokens, heads, pairs, p, addr(out),
                                              L.DTYPES[out_dtype]))


def qknorm_rope_peers(graph: Graph, x, weight, cos, sin, tokens: int, heads: int, dst: list, row0: int, eps=1e-5,
                      offset=1.0, pairing="interleaved") -> None:
    """qknorm_rope on bf16 rows of 128-wide heads, each output row stored straight into the memory of the rank that
    attends its head (we_qknorm_rope_peers): dst[r] is rank r's [world x tokens, heads / world, 128] block (a device
    address), this rank's rows starting at row row0 of it."""
    p = L.ROPE_HALF if pairing == "half" else L.ROPE_INTERLEAVED
    table = (C.c_void_p * len(dst))(*dst)
    L.check(graph.ctx, L.lib().we_qknorm_rope_peers(graph.ctx, addr(x), addr(weight), eps, offset, addr(cos),
                                                    addr(sin), tokens, heads, p, table, len(dst), row0))


def quantize_fp8(graph: Graph, w, n: int, k: int, q, scales, per_channel: bool = True, w_dtype="f32") -> None:
    L.check(graph.ctx, L.lib().we_quantize_fp8(graph.ctx, addr(w), L.DTYPES[w_dtype], n, k, int(per_channel), addr(q),
                                               addr(scales)))


def quantize_int4(graph: Graph, w, n: int, k: int, packed, scales, w_dtype="f32") -> None:
    L.check(graph.ctx, L.lib().we_quantize_int4(graph.ctx, addr(w), L.DTYPES[w_dtype], n, k, addr(packed),
                                                addr(scales)))


def quantize_act(graph: Graph, x, m: int, k: int, hi, lo, row_scale, terms: int = 2, x_stride: int = 0,
                 x_dtype="bf16") -> None:
    L.check(graph.ctx, L.lib().we_quantize_act(graph.ctx, addr(x), L.DTYPES[x_dtype], m, k, x_stride, terms, addr(hi),
                                               addr(lo), addr(row_scale)))


def gemm_fp8(graph: Graph, x_hi, x_lo, row_scale, w, y, m: int, n: int, k: int, scale: float = 1.0,
             chan_scale=None, bias=None, y_dtype="f32", y_stride: int = 0, accumulate: bool = False,
             act=None, aux_op=None, aux=None, aux_dtype="f32", gate=None, parts=None, set2=None,
             segments=None, peer=None) -> None:
    """The tcgen05 GEMM on an already-split activation (we_gemm_fp8); x_lo None = one term. parts: a split output,
    [(buffer, width), ...] taking the channels in order (y is then unused). set2 / segments: a second weight set,
    set2 = dict(w=, scale=, chan_scale=, bias=, gate=) used by the row segments marked 1 in segments =
    [(row_end, set), ...]. peer = dict(dst=[address per rank], part=i, row0=r): part i (the whole output without
    parts) goes head by head straight into the ranks that attend its heads (we_gemm_fp8_desc.peer_dst)."""
    d = L.GemmFp8Desc(m, n, k, addr(x_hi).value, addr(x_lo).value, addr(row_scale).value, addr(w).value, scale,
                      addr(chan_scale).value, addr(bias).value, addr(y).value, y_stride, L.DTYPES[y_dtype],
                      L.MM_ACCUMULATE if accumulate else 0, epilogue(act, aux_op, aux, aux_dtype, gate))
    if parts:
        for i, (pt, width) in enumerate(parts):
            d.y_parts[i] = addr(pt).value
            d.part_n[i] = width
    if segments:
        s2 = set2 or {}
        d.w2, d.scale2 = addr(s2.get("w")).value, s2.get("scale", 1.0)
        d.chan_scale2, d.bias2, d.gate2 = (addr(s2.get(x)).value for x in ("chan_scale", "bias", "gate"))
        d.nseg = len(segments)
        for i, (end, st) in enumerate(segments):
            d.row_end[i], d.row_set[i] = end, st
    if peer:
        for r, a in enumerate(peer["dst"]):
            d.peer_dst[r] = a
        d.peer_world, d.peer_part, d.peer_row0 = len(peer["dst"]), peer.get("part", 0), peer["row0"]
    L.check(graph.ctx, L.lib().we_gemm_fp8(graph.ctx, C.byref(d)))


def unpack_fp8_bf16(graph: Graph, data, n: int, out) -> None:
    L.check(graph.ctx, L.lib().we_unpack_fp8_bf16(graph.ctx, addr(data), n, addr(out)))


def unpack_int4(graph: Graph, packed, scales, n: int, k: int, out) -> None:
    L.check(graph.ctx, L.lib().we_unpack_int4(graph.ctx, addr(packed), addr(scales), n, k, addr(out)))


def attention(graph: Graph, q, k, v, tokens: int, heads: int, kv_heads: int, dim: int, out, causal: bool = False,
              dtype: str = "f32", out_dtype: str = "f32") -> None:
    """attention into a given output buffer (src/kernels/attention.ts:20-51)."""
    L.check(graph.ctx, L.lib().we_attention(graph.ctx, addr(q), addr(k), addr(v), L.DTYPES[dtype], tokens, heads,
                                            kv_heads, dim, int(causal), addr(out), L.DTYPES[out_dtype]))


def norm_split(graph: Graph, x, weight, rows: int, d: int, hi, lo, row_scale, scale=None, shift=None, eps=1e-5,
               offset=1.0, terms: int = 2, x_dtype: str = "f32") -> None:
    """RMSNorm + modulation, rounded to bf16 and split into e4m3 planes for the fp8 GEMM, in one pass."""
    L.check(graph.ctx, L.lib().we_norm_split(graph.ctx, addr(x), L.DTYPES[x_dtype], addr(weight), addr(scale),
                                             addr(shift), rows, d, eps, offset, terms, addr(hi), addr(lo),
                                             addr(row_scale)))


def add_norm_split(graph: Graph, x, r, xo, weight, rows: int, d: int, hi, lo, row_scale, scale=None, shift=None,
                   eps=1e-5, offset=1.0, terms: int = 2) -> None:
    """xo = x + r (f32), then norm + split of xo (we_add_norm_split): a block's residual add fused with the next
    RMSNorm and activation split."""
    L.check(graph.ctx, L.lib().we_add_norm_split(graph.ctx, addr(x), addr(r), addr(xo), addr(weight), addr(scale),
                                                 addr(shift), rows, d, eps, offset, terms, addr(hi), addr(lo),
                                                 addr(row_scale)))
