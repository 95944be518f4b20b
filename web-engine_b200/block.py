"""One transformer block on the hot-path kernels: the caller of linear / norm / rotate (src/model/block.ts).

    h  = (1 + prescale) norm1(x) + preshift
    x1 = x + pregate  wo(attention(rope(norm_q(wq h)), rope(norm_k(wk h)), wv h) [ * sigmoid(gate h)])
    h2 = (1 + postscale) norm2(x1) + postshift
    y  = x1 + postgate down(mlp(h2)),  mlp = silu(mlp_gate h2) up h2 (Krea 2)  or  gelu(up h2)

`block(..., dtype="f32")` mirrors block.ts op by op (linear, norm, rotate, attention, sigmoidGate, gatedAdd,
swiglu: the reference's f32 semantics, src/model/block.ts:91-105). `dtype="bf16"` is the B200 path:
- each RMSNorm writes the e4m3 split of its bf16 output directly (we_norm_split) for the fp8 GEMMs;
- q/k get the fused norm + RoPE;
- attention runs on the tcgen05 flash kernel;
- the sigmoid gate, the MLP activation and the gated residual adds run inside the GEMM epilogues.
The residual stream stays f32.
"""
from __future__ import annotations

from dataclasses import dataclass

from . import kernels as K
from . import ops
from .graph import Buffer, Graph


@dataclass
class BlockConfig:
    """BlockConfig (src/model/block.ts:6-8) plus the MLP kind and whether attention has a sigmoid gate."""

    hidden: int
    mlp: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float = 1e-5
    mlp_act: str = "swiglu"   # "swiglu" (Krea 2) | "gelu"
    attn_gate: bool = True


@dataclass
class BlockWeights:
    """Device weights of one block. Linears are ops.Linear (fp8 with per-tensor or per-channel scales);
    norm weights and the modulation table are f32."""

    wq: ops.Linear
    wk: ops.Linear
    wv: ops.Linear
    wo: ops.Linear
    mlp_up: ops.Linear
    mlp_down: ops.Linear
    norm1: object
    norm2: object
    norm_q: object
    norm_k: object
    table: object            # [6 * hidden]
    gate: ops.Linear | None = None
    mlp_gate: ops.Linear | None = None


MOD = ("prescale", "preshift", "pregate", "postscale", "postshift", "postgate")


def modulation(graph: Graph, tvec, table, hidden: int) -> dict:
    """tvec + the block's table, split into the 6 modulation vectors (src/model/block.ts:33-37)."""
    mod = ops.add(graph, tvec, table, 6 * hidden)
    return {name: Graph.slice(mod, i * hidden * 4, hidden * 4) if (i * hidden * 4) % 256 == 0
            else _Offset(mod, i * hidden * 4) for i, name in enumerate(MOD)}


class _Offset:
    """A device address inside a buffer, for slices not on a 256-byte boundary."""

    def __init__(self, buf: Buffer, offset: int):
        self.ptr = buf.ptr + offset

    @property
    def c(self):
        import ctypes

        return ctypes.c_void_p(self.ptr)


def block(graph: Graph, w: BlockWeights, cfg: BlockConfig, x, tvec, rope: ops.Rope, dtype: str = "f32") -> Buffer:
    """x [tokens, hidden] f32 -> a new [tokens, hidden] f32 buffer."""
    if dtype == "f32":
        return _block_f32(graph, w, cfg, x, tvec, rope)
    if dtype == "bf16":
        return _block_bf16(graph, w, cfg, x, tvec, rope)
    raise ValueError(f"unknown block dtype {dtype}")


def _block_f32(graph, w, cfg, x, tvec, rope):
    t, hd = rope.tokens, cfg.hidden
    mark = graph.mark()
    mod = modulation(graph, tvec, w.table, hd)
    h = ops.norm(graph, x, w.norm1, t, hd, ops.Mod(mod["prescale"], mod["preshift"]), cfg.eps)
    none = ops.no_mod(graph, cfg.head_dim)
    q = ops.linear(graph, h, w.wq, t)
    q = ops.norm(graph, q, w.norm_q, t * cfg.heads, cfg.head_dim, none, cfg.eps)
    q = ops.rotate(graph, q, cfg.heads, rope)
    k = ops.linear(graph, h, w.wk, t)
    k = ops.norm(graph, k, w.norm_k, t * cfg.kv_heads, cfg.head_dim, none, cfg.eps)
    k = ops.rotate(graph, k, cfg.kv_heads, rope)
    v = ops.linear(graph, h, w.wv, t)
    o = ops.attention(graph, q, k, v, t, cfg.heads, cfg.kv_heads, cfg.head_dim)
    if cfg.attn_gate:
        g = ops.linear(graph, h, w.gate, t)
        o = ops.sigmoid_gate(graph, o, g, t * hd)
    a = ops.linear(graph, o, w.wo, t)
    x1 = ops.gated_add(graph, x, a, mod["pregate"], t * hd, hd)
    h2 = ops.norm(graph, x1, w.norm2, t, hd, ops.Mod(mod["postscale"], mod["postshift"]), cfg.eps)
    if cfg.mlp_act == "swiglu":
        m = ops.swiglu(graph, ops.linear(graph, h2, w.mlp_gate, t), ops.linear(graph, h2, w.mlp_up, t), t * cfg.mlp)
    else:
        m = ops.gelu(graph, ops.linear(graph, h2, w.mlp_up, t), t * cfg.mlp)
    d = ops.linear(graph, m, w.mlp_down, t)
    out = ops.gated_add(graph, x1, d, mod["postgate"], t * hd, hd)
    graph.release(mark, [out])
    return out


def _gemm(graph, split, lin: ops.Linear, y, t, y_dtype, **epi):
    hi, lo, rs = split
    K.gemm_fp8(graph, hi, lo, rs, lin.buffer, y, t, lin.n, lin.k, lin.scale, chan_scale=lin.chan_scale,
               bias=lin.bias, y_dtype=y_dtype, **epi)


def _block_bf16(graph, w, cfg, x, tvec, rope):
    t, hd, hdim = rope.tokens, cfg.hidden, cfg.head_dim
    mark = graph.mark()
    mod = modulation(graph, tvec, w.table, hd)
    split = (graph.buffer(t * hd), graph.buffer(t * hd), graph.buffer(t * 4))
    K.norm_split(graph, x, w.norm1, t, hd, *split, scale=mod["prescale"], shift=mod["preshift"], eps=cfg.eps)
    q = graph.buffer(t * cfg.heads * hdim * 2)
    k = graph.buffer(t * cfg.kv_heads * hdim * 2)
    v = graph.buffer(t * cfg.kv_heads * hdim * 2)
    _gemm(graph, split, w.wq, q, t, "bf16")
    _gemm(graph, split, w.wk, k, t, "bf16")
    _gemm(graph, split, w.wv, v, t, "bf16")
    K.qknorm_rope(graph, q, w.norm_q, rope.cos, rope.sin, t, cfg.heads, rope.pairs, q, eps=cfg.eps,
                  x_dtype="bf16", out_dtype="bf16")
    K.qknorm_rope(graph, k, w.norm_k, rope.cos, rope.sin, t, cfg.kv_heads, rope.pairs, k, eps=cfg.eps,
                  x_dtype="bf16", out_dtype="bf16")
    o = graph.buffer(t * hd * 2)
    K.attention(graph, q, k, v, t, cfg.heads, cfg.kv_heads, hdim, o, dtype="bf16", out_dtype="bf16")
    if cfg.attn_gate:  # og = o * sigmoid(gate h), in the gate GEMM's epilogue
        og = graph.buffer(t * hd * 2)
        _gemm(graph, split, w.gate, og, t, "bf16", aux_op="sigmoid_gate", aux=o, aux_dtype="bf16")
        o = og
    K.quantize_act(graph, o, t, hd, *split, terms=2)
    x1 = graph.buffer(t * hd * 4)
    graph.copy(x, 0, x1, 0, t * hd * 4)
    _gemm(graph, split, w.wo, x1, t, "f32", accumulate=True, gate=mod["pregate"])  # x1 = x + pregate wo(o)
    K.norm_split(graph, x1, w.norm2, t, hd, *split, scale=mod["postscale"], shift=mod["postshift"], eps=cfg.eps)
    u = graph.buffer(t * cfg.mlp * 2)
    if cfg.mlp_act == "swiglu":
        g = graph.buffer(t * cfg.mlp * 2)
        _gemm(graph, split, w.mlp_gate, g, t, "bf16")
        _gemm(graph, split, w.mlp_up, u, t, "bf16", aux_op="swiglu", aux=g, aux_dtype="bf16")
    else:
        _gemm(graph, split, w.mlp_up, u, t, "bf16", act="gelu_tanh")
    msplit = (graph.buffer(t * cfg.mlp), graph.buffer(t * cfg.mlp), split[2])
    K.quantize_act(graph, u, t, cfg.mlp, *msplit, terms=2)
    out = graph.buffer(t * hd * 4)
    graph.copy(x1, 0, out, 0, t * hd * 4)
    _gemm(graph, msplit, w.mlp_down, out, t, "f32", accumulate=True, gate=mod["postgate"])  # out = x1 + postgate d
    graph.release(mark, [out])
    return out


def block_flops(cfg: BlockConfig, tokens: int) -> dict:
    """Multiply-add work of one block (2 FLOP per MAC): linears and attention (4 T^2 H D)."""
    hd, kvd = cfg.hidden, cfg.kv_heads * cfg.head_dim
    lin = 2 * tokens * (hd * hd * (2 + (1 if cfg.attn_gate else 0)) + 2 * hd * kvd
                        + hd * cfg.mlp * (3 if cfg.mlp_act == "swiglu" else 2))
    attn = 4 * tokens * tokens * cfg.heads * cfg.head_dim
    return {"linear": lin, "attention": attn, "total": lin + attn}
