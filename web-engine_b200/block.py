"""Transformer blocks on the hot-path kernels: the callers of linear / norm / rotate (src/model/block.ts).

A single-stream block (block.ts:83-105):

    h  = (1 + prescale) norm1(x) + preshift
    x1 = x + pregate  wo(attention(rope(norm_q(wq h)), rope(norm_k(wk h)), wv h) [ * sigmoid(gate h)])
    h2 = (1 + postscale) norm2(x1) + postshift
    y  = x1 + postgate down(mlp(h2)),  mlp = silu(mlp_gate h2) up h2 (Krea 2)  or  gelu(up h2) (GELU MLP)

A double-stream block runs the same formulas on two row ranges of one token sequence (text rows first, then
image rows), each with its own weights and modulation table, and one attention over all rows (the Flux-style
MMDiT block; every op it uses is the single block's). Both are `joint_block` over a list of `Part`s.

`dtype="f32"` mirrors block.ts op by op (linear, norm, rotate, attention, sigmoidGate, gatedAdd, swiglu: the
reference's f32 semantics, src/model/block.ts:91-105). `dtype="bf16"` is the B200 path:
- each RMSNorm writes the e4m3 split of its bf16 output directly (we_norm_split) for the fp8 GEMMs;
- q/k get the fused norm + RoPE;
- attention runs on the tcgen05 flash kernel;
- the sigmoid gate, the MLP activation and the residual gates run inside the GEMM epilogues; the first residual
  add is fused with the second RMSNorm + split (we_add_norm_split), the second is one f32 add, or, when the
  caller chains blocks (`defer=True`), is left to the next block's first RMSNorm + split (a `Residual`).
The residual stream stays f32.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import kernels as K
from . import ops
from .graph import Buffer, Graph, addr


@dataclass
class Residual:
    """A bf16 block's output y = x1 + dn with the add not yet done: the next block's first norm pass adds the two
    (we_add_norm_split), which saves the add's launch and one read of y. Both buffers are the caller's."""

    x1: Buffer
    dn: Buffer

    def buffers(self) -> list:
        return [self.x1, self.dn]


def buffers_of(x) -> list:
    """The graph buffers that hold a block's output (one Buffer, or a Residual's two)."""
    return x.buffers() if isinstance(x, Residual) else [x]


@dataclass
class BlockConfig:
    """BlockConfig (src/model/block.ts:6-8) plus the MLP kind and whether attention has a sigmoid gate."""

    hidden: int
    mlp: int
    heads: int
    kv_heads: int
    head_dim: int
    eps: float = 1e-5
    mlp_act: str = "swiglu"   # "swiglu" (Krea 2) | "gelu" (tanh GELU, 4x MLP)
    attn_gate: bool = True

    def __post_init__(self):
        # attention's output is rows x hidden (sigmoidGate over rows * hidden, wo [hidden, hidden]: block.ts:61-64)
        if self.heads * self.head_dim != self.hidden:
            raise ValueError(f"heads x head_dim ({self.heads} x {self.head_dim}) must equal hidden ({self.hidden})")
        if self.kv_heads <= 0 or self.heads % self.kv_heads:
            raise ValueError("heads must be a multiple of kvHeads")
        if self.mlp_act not in ("swiglu", "gelu"):
            raise ValueError(f"unknown MLP activation {self.mlp_act}")


@dataclass
class BlockWeights:
    """Device weights of one block (or one stream of a double block). Linears are ops.Linear (fp8 with
    per-tensor or per-channel scales); norm weights and the modulation table are f32."""

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
    wqkv: ops.Linear | None = None  # [wq; wk; wv] in one buffer (fuse_qkv): one GEMM for the three projections


def fuse_qkv(graph: Graph, w: BlockWeights) -> BlockWeights:
    """Adds w.wqkv: the q, k and v weights concatenated along the output channels with their per-channel scales
    (a scalar scale becomes a constant run) and biases, so the bf16 path runs one GEMM whose epilogue writes q, k
    and v to their own buffers. Three N = 3072 GEMMs fill the GPU poorly (at 2304 tokens, 108 tiles for 74 SM
    pairs: 176 us); one N = 9216 GEMM takes 107 us. Needs fp8 weights with the same K and part boundaries at
    multiples of 32 channels; otherwise w is returned unchanged. The fused copy is extra memory (n x k bytes);
    call it where the weights are created, outside any mark / release scope."""
    lins = (w.wq, w.wk, w.wv)
    if w.wqkv is not None or any(l.dtype != "fp8" or l.k != w.wq.k or l.lora is not None for l in lins):
        return w
    if w.wq.n % 32 or (w.wq.n + w.wk.n) % 32:
        return w
    k, n = w.wq.k, sum(l.n for l in lins)
    buf = graph.buffer(n * k)
    scales = graph.buffer(n * 4)
    bias = graph.buffer(n * 4) if any(l.bias is not None for l in lins) else None
    off = 0
    temps = []
    for l in lins:
        graph.copy(l.buffer, 0, buf, off * k, l.n * k)
        sc = l.chan_scale
        if sc is None:
            sc = graph.buffer(np.full(l.n, l.scale, np.float32))
            temps.append(sc)
        graph.copy(sc, 0, scales, off * 4, l.n * 4)
        if bias is not None:
            b = l.bias
            if b is None:
                b = graph.buffer(l.n * 4)  # zeros
                temps.append(b)
            graph.copy(b, 0, bias, off * 4, l.n * 4)
        off += l.n
    for t in temps:  # stream-ordered: the pool hands them out again only after the copies
        graph.free(t)
    w.wqkv = ops.Linear(buf, "fp8", 1.0, n, k, bias=bias, chan_scale=scales)
    return w


@dataclass
class Part:
    """Rows [row0, row0 + rows) of the token sequence, with their own block weights."""

    row0: int
    rows: int
    w: BlockWeights


MOD = ("prescale", "preshift", "pregate", "postscale", "postshift", "postgate")


def modulation(graph: Graph, tvec, table, hidden: int) -> dict:
    """tvec + the block's table, split into the 6 modulation vectors (src/model/block.ts:33-37)."""
    mod = ops.add(graph, tvec, table, 6 * hidden)
    return {name: mod.ptr + i * hidden * 4 for i, name in enumerate(MOD)}


def rows_at(buf, row0: int, row_bytes: int) -> int:
    """Device address of row `row0` of a row-major buffer."""
    return addr(buf).value + row0 * row_bytes


def part_rope(rope: ops.Rope, p: Part) -> ops.Rope:
    """The cos/sin rows of one part."""
    return ops.Rope(rows_at(rope.cos, p.row0, rope.pairs * 4), rows_at(rope.sin, p.row0, rope.pairs * 4), rope.pairs,
                    p.rows)


def block(graph: Graph, w: BlockWeights, cfg: BlockConfig, x, tvec, rope: ops.Rope, dtype: str = "f32") -> Buffer:
    """A single-stream block: x [tokens, hidden] f32 -> a new [tokens, hidden] f32 buffer."""
    return joint_block(graph, [Part(0, rope.tokens, w)], cfg, x, tvec, rope, dtype)


def double_block(graph: Graph, txt: BlockWeights, img: BlockWeights, cfg: BlockConfig, x, txt_rows: int, tvec,
                 rope: ops.Rope, dtype: str = "f32") -> Buffer:
    """A double-stream block: rows [0, txt_rows) use `txt`, the rest `img`; attention spans all rows."""
    return joint_block(graph, [Part(0, txt_rows, txt), Part(txt_rows, rope.tokens - txt_rows, img)], cfg, x, tvec, rope,
                       dtype)


@dataclass
class TPLayer:
    """What a tensor-parallel block needs beyond its local rows: the communicator of the group, the layer's parts
    over all T rows of the image (global row offsets; the weights are this rank's shards) and the RoPE tables of
    all T rows."""

    comm: object
    parts_all: list
    rope_all: ops.Rope


def joint_block(graph: Graph, parts: list, cfg: BlockConfig, x, tvec, rope: ops.Rope, dtype: str = "f32",
                images: int = 1, sp=None, defer: bool = False, tp: TPLayer | None = None):
    """Rows of `images` sequences of rope.tokens / images tokens each, stacked; each part covers a row range with its
    own weights, attention runs within each image. rope: cos/sin for all stacked rows (per image, tiled).
    sp: a sequence.SequenceParallel when the rows are this rank's shard of one image (bf16 path).
    x: a Buffer [tokens, hidden] f32 or the Residual a previous block deferred. defer: on the bf16 path, return
    the output as a Residual for the next block instead of adding it here (the f32 path always returns a Buffer)."""
    parts = [p for p in parts if p.rows > 0]
    if sum(p.rows for p in parts) != rope.tokens:
        raise ValueError("the parts must cover the rope's tokens")
    if images < 1 or rope.tokens % images:
        raise ValueError("the rows must split evenly into images")
    if sp is not None and (dtype != "bf16" or images != 1):
        raise ValueError("a sequence-parallel block runs one image on the bf16 path")
    if tp is not None:
        if dtype != "bf16" or images != 1 or sp is not None:
            raise ValueError("a tensor-parallel block runs one image on the bf16 path")
        return _joint_bf16_tp(graph, parts, cfg, x, tvec, tp, defer)
    if dtype == "f32":
        if isinstance(x, Residual):
            x = ops.add(graph, x.x1, x.dn, rope.tokens * cfg.hidden)
        return _joint_f32(graph, parts, cfg, x, tvec, rope, images)
    if dtype == "bf16":
        return _joint_bf16(graph, parts, cfg, x, tvec, rope, images, sp, defer)
    raise ValueError(f"unknown block dtype {dtype}")


def _attend_sp(graph, sp, q, k, v, t: int, cfg: BlockConfig):
    """Attention of one image whose rows are sharded over sp's ranks: q/k/v go token shard -> head shard, this
    rank attends heads / world heads over every token, the output comes back the same way. Returns this rank's
    output rows [t, heads x 128] (bf16): in sp's peer region on the peer path, a graph buffer on the nccl one."""
    hb, T = cfg.head_dim * 2, t * sp.world
    hl, kl = cfg.heads // sp.world, cfg.kv_heads // sp.world
    if sp.peer:
        def attend(qh, kh, vh, oh):
            K.attention(graph, qh, kh, vh, T, hl, kl, cfg.head_dim, oh, dtype="bf16", out_dtype="bf16")

        return sp.exchange_heads(graph, q, k, v, t, cfg.heads, cfg.kv_heads, hb, attend)
    o = graph.buffer(t * cfg.hidden * 2)
    qh = sp.scatter_heads(graph, q, t, cfg.heads, hb, "q")
    kh = sp.scatter_heads(graph, k, t, cfg.kv_heads, hb, "k")
    vh = sp.scatter_heads(graph, v, t, cfg.kv_heads, hb, "v")
    oh = sp.buffer("o_heads", T * hl * hb)
    K.attention(graph, qh, kh, vh, T, hl, kl, cfg.head_dim, oh, dtype="bf16", out_dtype="bf16")
    sp.gather_heads(graph, oh, t, cfg.heads, hb, o)
    return o


def _attend_images(graph, q, k, v, o, rows: int, cfg: BlockConfig, images: int, dtype: str) -> None:
    """Attention of each image's rows into o (one launch per image)."""
    t = rows // images
    qw, kw = cfg.heads * cfg.head_dim, cfg.kv_heads * cfg.head_dim
    es = 2 if dtype == "bf16" else 4
    for i in range(images):
        K.attention(graph, rows_at(q, i * t, qw * es), rows_at(k, i * t, kw * es), rows_at(v, i * t, kw * es), t,
                    cfg.heads, cfg.kv_heads, cfg.head_dim, rows_at(o, i * t, qw * es), dtype=dtype, out_dtype=dtype)


def _joint_f32(graph, parts, cfg, x, tvec, rope, images=1):
    t, hd, hdim = rope.tokens, cfg.hidden, cfg.head_dim
    qw, kw = cfg.heads * hdim, cfg.kv_heads * hdim
    mark = graph.mark()
    none = ops.no_mod(graph, hdim)
    one = len(parts) == 1
    if not one:
        q, k, v = graph.buffer(t * qw * 4), graph.buffer(t * kw * 4), graph.buffer(t * kw * 4)
    hs, mods = [], []
    for p in parts:
        mod = modulation(graph, tvec, p.w.table, hd)
        h = ops.norm(graph, rows_at(x, p.row0, hd * 4), p.w.norm1, p.rows, hd,
                     ops.Mod(mod["prescale"], mod["preshift"]), cfg.eps)
        pr = part_rope(rope, p)
        qp = ops.linear(graph, h, p.w.wq, p.rows)
        qp = ops.rotate(graph, ops.norm(graph, qp, p.w.norm_q, p.rows * cfg.heads, hdim, none, cfg.eps), cfg.heads, pr)
        kp = ops.linear(graph, h, p.w.wk, p.rows)
        kp = ops.rotate(graph, ops.norm(graph, kp, p.w.norm_k, p.rows * cfg.kv_heads, hdim, none, cfg.eps),
                        cfg.kv_heads, pr)
        vp = ops.linear(graph, h, p.w.wv, p.rows)
        if one:
            q, k, v = qp, kp, vp
        else:
            graph.copy(qp, 0, q, p.row0 * qw * 4, p.rows * qw * 4)
            graph.copy(kp, 0, k, p.row0 * kw * 4, p.rows * kw * 4)
            graph.copy(vp, 0, v, p.row0 * kw * 4, p.rows * kw * 4)
        hs.append(h)
        mods.append(mod)
    if images == 1:
        o = ops.attention(graph, q, k, v, t, cfg.heads, cfg.kv_heads, hdim)
    else:
        o = graph.buffer(t * qw * 4)
        _attend_images(graph, q, k, v, o, t, cfg, images, "f32")
    out = None if one else graph.buffer(t * hd * 4)
    for p, h, mod in zip(parts, hs, mods):
        op = rows_at(o, p.row0, hd * 4)
        if cfg.attn_gate:
            op = ops.sigmoid_gate(graph, op, ops.linear(graph, h, p.w.gate, p.rows), p.rows * hd)
        a = ops.linear(graph, op, p.w.wo, p.rows)
        x1 = ops.gated_add(graph, rows_at(x, p.row0, hd * 4), a, mod["pregate"], p.rows * hd, hd)
        h2 = ops.norm(graph, x1, p.w.norm2, p.rows, hd, ops.Mod(mod["postscale"], mod["postshift"]), cfg.eps)
        if cfg.mlp_act == "swiglu":
            m = ops.swiglu(graph, ops.linear(graph, h2, p.w.mlp_gate, p.rows), ops.linear(graph, h2, p.w.mlp_up, p.rows),
                           p.rows * cfg.mlp)
        else:
            m = ops.gelu(graph, ops.linear(graph, h2, p.w.mlp_up, p.rows), p.rows * cfg.mlp)
        d = ops.linear(graph, m, p.w.mlp_down, p.rows)
        op_out = ops.gated_add(graph, x1, d, mod["postgate"], p.rows * hd, hd)
        if one:
            out = op_out
        else:
            graph.copy(op_out, 0, out, p.row0 * hd * 4, p.rows * hd * 4)
    graph.release(mark, [out])
    return out


def _weight_plan(parts, t: int):
    """How a block's linears run over its parts: ("one", w) when one weight set covers rows [0, t) (one GEMM);
    ("two", segments, w0, w1) when two weight sets tile [0, t) in row segments at multiples of 64 (one GEMM whose
    token tiles pick their weights: a double block's text and image rows, for every image of a batch); None: one
    GEMM per part."""
    end = 0
    for p in parts:
        if p.row0 != end:
            return None
        end += p.rows
    if end != t:
        return None
    ws: list = []
    for p in parts:
        if not any(p.w is w for w in ws):
            ws.append(p.w)
    if len(ws) == 1:
        return ("one", ws[0])
    if len(ws) != 2:
        return None
    segs: list = []
    for p in parts:
        st = 0 if p.w is ws[0] else 1
        if segs and segs[-1][1] == st:
            segs[-1] = (p.row0 + p.rows, st)
        else:
            segs.append((p.row0 + p.rows, st))
    if len(segs) > 32 or any(e % 64 for e, _ in segs[:-1]):
        return None
    return ("two", segs, ws[0], ws[1])


def _gemm_all(graph, plan, parts, split, width: int, lin, outs, y_dtype: str, mods=None, gate_key=None, aux=None,
              aux_row_bytes: int = 0, peer=None, **epi):
    """The linear lin(w) of every part, over all rows: split holds the e4m3 planes of rows [0, t) (width values a
    row), outs = [(buffer, channels), ...] the output rows (one buffer, or the q / k / v parts of a split output),
    mods[id(w)][gate_key] the per-channel gate of a weight set, aux an epilogue operand over all rows. peer =
    dict(dst=, part=, row0=): that output part goes to the ranks that attend its heads (gemm_fp8's peer), row 0 of
    these rows at row row0 of their blocks."""
    es = 2 if y_dtype == "bf16" else 4

    def call(sr, rows, w, ys, aux_p, row_ofs=0, **more):
        ln = lin(w)
        gate = mods[id(w)][gate_key] if gate_key else None
        y, pt = (ys[0][0], None) if len(ys) == 1 else (None, ys)
        pe = dict(peer, row0=peer["row0"] + row_ofs) if peer else None
        K.gemm_fp8(graph, *sr, ln.buffer, y, rows, ln.n, ln.k, ln.scale, chan_scale=ln.chan_scale, bias=ln.bias,
                   y_dtype=y_dtype, gate=gate, aux=aux_p, parts=pt, peer=pe, **epi, **more)

    if plan is not None and plan[0] == "one":
        call(split, parts[-1].row0 + parts[-1].rows, plan[1], outs, aux)
    elif plan is not None:
        _, segs, w0, w1 = plan
        l1 = lin(w1)
        set2 = dict(w=l1.buffer, scale=l1.scale, chan_scale=l1.chan_scale, bias=l1.bias,
                    gate=mods[id(w1)][gate_key] if gate_key else None)
        call(split, segs[-1][0], w0, outs, aux, set2=set2, segments=segs)
    else:
        for p in parts:
            call(_split_rows(split, p, width), p.rows, p.w, [(rows_at(b, p.row0, n * es), n) for b, n in outs],
                 rows_at(aux, p.row0, aux_row_bytes) if aux is not None else None, p.row0)


def _split_rows(split, p: Part, width: int):
    """The e4m3 planes (1 byte per value) and row scales of one part."""
    return (rows_at(split[0], p.row0, width), rows_at(split[1], p.row0, width), rows_at(split[2], p.row0, 4))


def _joint_bf16(graph, parts, cfg, x, tvec, rope, images=1, sp=None, defer=False):
    t, hd, hdim = rope.tokens, cfg.hidden, cfg.head_dim
    qw, kw = cfg.heads * hdim, cfg.kv_heads * hdim
    mark = graph.mark()
    res = None
    if isinstance(x, Residual):  # x = x1 + dn of the previous block, written by the first norm pass below
        res, x = x, graph.buffer(t * hd * 4)
    shared: dict = {}  # parts with the same weights (the images of a batch) share one modulation
    mods = []
    for p in parts:
        if id(p.w) not in shared:
            shared[id(p.w)] = modulation(graph, tvec, p.w.table, hd)
        mods.append(shared[id(p.w)])
    plan = _weight_plan(parts, t)
    split = (graph.buffer(t * hd), graph.buffer(t * hd), graph.buffer(t * 4))
    q, k, v = graph.buffer(t * qw * 2), graph.buffer(t * kw * 2), graph.buffer(t * kw * 2)
    for p, mod in zip(parts, mods):
        if res is None:
            K.norm_split(graph, rows_at(x, p.row0, hd * 4), p.w.norm1, p.rows, hd, *_split_rows(split, p, hd),
                         scale=mod["prescale"], shift=mod["preshift"], eps=cfg.eps)
        else:
            K.add_norm_split(graph, rows_at(res.x1, p.row0, hd * 4), rows_at(res.dn, p.row0, hd * 4),
                             rows_at(x, p.row0, hd * 4), p.w.norm1, p.rows, hd, *_split_rows(split, p, hd),
                             scale=mod["prescale"], shift=mod["preshift"], eps=cfg.eps)
    # sequence parallelism, fused exchange: the q/k/v GEMM's epilogue stores v, and q / k norm + RoPE store q and k,
    # straight into the regions of the ranks that attend their heads (no copy kernel after them)
    tg = None
    if sp is not None and sp.fused and hdim == 128:
        tg = sp.head_targets(graph, t, cfg.heads, cfg.kv_heads, hdim * 2)
    vpeer = dict(dst=tg["v"], row0=tg["row0"]) if tg else None
    if all(p.w.wqkv is not None for p in parts):  # one GEMM, its epilogue writing q, k and v
        _gemm_all(graph, plan, parts, split, hd, lambda w: w.wqkv, [(q, qw), (k, kw), (v, kw)], "bf16",
                  peer=dict(vpeer, part=2) if vpeer else None)
    else:
        for name, buf, n in (("wq", q, qw), ("wk", k, kw), ("wv", v, kw)):
            _gemm_all(graph, plan, parts, split, hd, lambda w, nm=name: getattr(w, nm), [(buf, n)], "bf16",
                      peer=dict(vpeer, part=0) if vpeer and name == "wv" else None)
    for p in parts:
        qp, kp = rows_at(q, p.row0, qw * 2), rows_at(k, p.row0, kw * 2)
        pr = part_rope(rope, p)
        if tg:
            K.qknorm_rope_peers(graph, qp, p.w.norm_q, pr.cos, pr.sin, p.rows, cfg.heads, tg["q"], tg["row0"] + p.row0,
                                eps=cfg.eps)
            K.qknorm_rope_peers(graph, kp, p.w.norm_k, pr.cos, pr.sin, p.rows, cfg.kv_heads, tg["k"],
                                tg["row0"] + p.row0, eps=cfg.eps)
            continue
        K.qknorm_rope(graph, qp, p.w.norm_q, pr.cos, pr.sin, p.rows, cfg.heads, rope.pairs, qp, eps=cfg.eps,
                      x_dtype="bf16", out_dtype="bf16")
        K.qknorm_rope(graph, kp, p.w.norm_k, pr.cos, pr.sin, p.rows, cfg.kv_heads, rope.pairs, kp, eps=cfg.eps,
                      x_dtype="bf16", out_dtype="bf16")
    if sp is None:
        o = graph.buffer(t * hd * 2)
        _attend_images(graph, q, k, v, o, t, cfg, images, "bf16")
    elif tg:
        hl, kl, T = cfg.heads // sp.world, cfg.kv_heads // sp.world, t * sp.world

        def attend(qh, kh, vh, oh):
            K.attention(graph, qh, kh, vh, T, hl, kl, hdim, oh, dtype="bf16", out_dtype="bf16")

        o = sp.finish_heads(graph, t, cfg.heads, hdim * 2, attend)
    else:
        o = _attend_sp(graph, sp, q, k, v, t, cfg)
    if cfg.attn_gate:  # og = o * sigmoid(gate h), in the gate GEMM's epilogue
        og = graph.buffer(t * hd * 2)
        _gemm_all(graph, plan, parts, split, hd, lambda w: w.gate, [(og, hd)], "bf16", aux=o, aux_row_bytes=hd * 2,
                  aux_op="sigmoid_gate", aux_dtype="bf16")
        o = og
    K.quantize_act(graph, o, t, hd, *split, terms=2)
    a = graph.buffer(t * hd * 4)  # a = pregate wo(o), the gate in the epilogue
    _gemm_all(graph, plan, parts, split, hd, lambda w: w.wo, [(a, hd)], "f32", shared, "pregate")
    x1 = graph.buffer(t * hd * 4)
    u = graph.buffer(t * cfg.mlp * 2)
    for p, mod in zip(parts, mods):  # x1 = x + a, and the norm + split of x1, in one pass
        K.add_norm_split(graph, rows_at(x, p.row0, hd * 4), rows_at(a, p.row0, hd * 4), rows_at(x1, p.row0, hd * 4),
                         p.w.norm2, p.rows, hd, *_split_rows(split, p, hd), scale=mod["postscale"],
                         shift=mod["postshift"], eps=cfg.eps)
    if cfg.mlp_act == "swiglu":
        g = graph.buffer(t * cfg.mlp * 2)
        _gemm_all(graph, plan, parts, split, hd, lambda w: w.mlp_gate, [(g, cfg.mlp)], "bf16")
        _gemm_all(graph, plan, parts, split, hd, lambda w: w.mlp_up, [(u, cfg.mlp)], "bf16", aux=g,
                  aux_row_bytes=cfg.mlp * 2, aux_op="swiglu", aux_dtype="bf16")
    else:
        _gemm_all(graph, plan, parts, split, hd, lambda w: w.mlp_up, [(u, cfg.mlp)], "bf16", act="gelu_tanh")
    msplit = (graph.buffer(t * cfg.mlp), graph.buffer(t * cfg.mlp), split[2])
    K.quantize_act(graph, u, t, cfg.mlp, *msplit, terms=2)
    dn = graph.buffer(t * hd * 4)  # dn = postgate down(m)
    _gemm_all(graph, plan, parts, msplit, cfg.mlp, lambda w: w.mlp_down, [(dn, hd)], "f32", shared, "postgate")
    if defer:  # the next block adds x1 + dn in its first norm pass
        graph.release(mark, [x1, dn])
        return Residual(x1, dn)
    out = ops.add(graph, x1, dn, t * hd)  # x1 + postgate down(m): the block's output
    graph.release(mark, [out])
    return out


def _joint_bf16_tp(graph, parts, cfg, x, tvec, tp: TPLayer, defer=False):
    """The bf16 block on this rank's token shard (parts: local rows) with its linears split over the ranks of
    tp.comm (Megatron-style: the linears of src/model/block.ts:53-64,74-81 split along N for q/k/v, gate and MLP up,
    along K for wo and MLP down):
      norm1 + split on local rows -> all-gather of the e4m3 planes and row scales -> q/k/v GEMM on this rank's
      heads (column shard) over all T rows -> q/k norm + RoPE -> attention of this rank's heads over every token ->
      [gate] -> split of o -> wo GEMM on this rank's K slice, f32 partial sums over all rows -> reduce-scatter to the
      local rows -> x1 = x + a fused with norm2 + split -> all-gather -> MLP up (column shard) + GELU -> split of u ->
      MLP down on this rank's K slice -> reduce-scatter.
    The weights in the parts are this rank's shards (parallel.shard_block). The gathered planes are the ones one GPU
    would compute, so the column-parallel outputs equal one GPU's channel for channel; the row-parallel GEMMs sum per
    rank partials in f32."""
    comm = tp.comm
    W = comm.world
    hd, hdim = cfg.hidden, cfg.head_dim
    if cfg.heads % W or cfg.kv_heads % W or cfg.mlp % W:
        raise ValueError(f"heads, kv heads and MLP width must split over {W} ranks")
    hl, kl, ml = cfg.heads // W, cfg.kv_heads // W, cfg.mlp // W
    qw, kw = hl * hdim, kl * hdim
    n = sum(p.rows for p in parts)
    T = n * W
    parts_all, rope = tp.parts_all, tp.rope_all
    if sum(p.rows for p in parts_all) != T or rope.tokens != T:
        raise ValueError("the layer's parts and RoPE tables must cover every rank's rows")
    mark = graph.mark()
    res = None
    if isinstance(x, Residual):
        res, x = x, graph.buffer(n * hd * 4)
    shared: dict = {}
    for p in parts_all:
        if id(p.w) not in shared:
            shared[id(p.w)] = modulation(graph, tvec, p.w.table, hd)
    mods = [shared[id(p.w)] for p in parts]
    plan = _weight_plan(parts_all, T)
    loc = (graph.buffer(n * hd), graph.buffer(n * hd), graph.buffer(n * 4))
    split = (graph.buffer(T * hd), graph.buffer(T * hd), graph.buffer(T * 4))

    def gather():
        comm.all_gather(loc[0], split[0], n * hd)
        comm.all_gather(loc[1], split[1], n * hd)
        comm.all_gather(loc[2], split[2], n * 4)

    for p, mod in zip(parts, mods):
        if res is None:
            K.norm_split(graph, rows_at(x, p.row0, hd * 4), p.w.norm1, p.rows, hd, *_split_rows(loc, p, hd),
                         scale=mod["prescale"], shift=mod["preshift"], eps=cfg.eps)
        else:
            K.add_norm_split(graph, rows_at(res.x1, p.row0, hd * 4), rows_at(res.dn, p.row0, hd * 4),
                             rows_at(x, p.row0, hd * 4), p.w.norm1, p.rows, hd, *_split_rows(loc, p, hd),
                             scale=mod["prescale"], shift=mod["preshift"], eps=cfg.eps)
    gather()
    q, k, v = graph.buffer(T * qw * 2), graph.buffer(T * kw * 2), graph.buffer(T * kw * 2)
    if all(p.w.wqkv is not None for p in parts_all):
        _gemm_all(graph, plan, parts_all, split, hd, lambda w: w.wqkv, [(q, qw), (k, kw), (v, kw)], "bf16")
    else:
        for name, buf, nn in (("wq", q, qw), ("wk", k, kw), ("wv", v, kw)):
            _gemm_all(graph, plan, parts_all, split, hd, lambda w, nm=name: getattr(w, nm), [(buf, nn)], "bf16")
    for p in parts_all:
        qp, kp = rows_at(q, p.row0, qw * 2), rows_at(k, p.row0, kw * 2)
        pr = part_rope(rope, p)
        K.qknorm_rope(graph, qp, p.w.norm_q, pr.cos, pr.sin, p.rows, hl, rope.pairs, qp, eps=cfg.eps,
                      x_dtype="bf16", out_dtype="bf16")
        K.qknorm_rope(graph, kp, p.w.norm_k, pr.cos, pr.sin, p.rows, kl, rope.pairs, kp, eps=cfg.eps,
                      x_dtype="bf16", out_dtype="bf16")
    o = graph.buffer(T * qw * 2)
    K.attention(graph, q, k, v, T, hl, kl, hdim, o, dtype="bf16", out_dtype="bf16")
    if cfg.attn_gate:  # this rank's gate channels are its heads' features
        og = graph.buffer(T * qw * 2)
        _gemm_all(graph, plan, parts_all, split, hd, lambda w: w.gate, [(og, qw)], "bf16", aux=o, aux_row_bytes=qw * 2,
                  aux_op="sigmoid_gate", aux_dtype="bf16")
        o = og
    osplit = (graph.buffer(T * qw), graph.buffer(T * qw), graph.buffer(T * 4))
    K.quantize_act(graph, o, T, qw, *osplit, terms=2)
    partial = graph.buffer(T * hd * 4)  # this rank's share of pregate wo(o), every row
    _gemm_all(graph, plan, parts_all, osplit, qw, lambda w: w.wo, [(partial, hd)], "f32", shared, "pregate")
    a = graph.buffer(n * hd * 4)
    comm.reduce_scatter(partial, a, n * hd, "f32")
    x1 = graph.buffer(n * hd * 4)
    for p, mod in zip(parts, mods):
        K.add_norm_split(graph, rows_at(x, p.row0, hd * 4), rows_at(a, p.row0, hd * 4), rows_at(x1, p.row0, hd * 4),
                         p.w.norm2, p.rows, hd, *_split_rows(loc, p, hd), scale=mod["postscale"],
                         shift=mod["postshift"], eps=cfg.eps)
    gather()
    u = graph.buffer(T * ml * 2)
    if cfg.mlp_act == "swiglu":
        gt = graph.buffer(T * ml * 2)
        _gemm_all(graph, plan, parts_all, split, hd, lambda w: w.mlp_gate, [(gt, ml)], "bf16")
        _gemm_all(graph, plan, parts_all, split, hd, lambda w: w.mlp_up, [(u, ml)], "bf16", aux=gt,
                  aux_row_bytes=ml * 2, aux_op="swiglu", aux_dtype="bf16")
    else:
        _gemm_all(graph, plan, parts_all, split, hd, lambda w: w.mlp_up, [(u, ml)], "bf16", act="gelu_tanh")
    msplit = (graph.buffer(T * ml), graph.buffer(T * ml), split[2])
    K.quantize_act(graph, u, T, ml, *msplit, terms=2)
    partial_dn = graph.buffer(T * hd * 4)
    _gemm_all(graph, plan, parts_all, msplit, ml, lambda w: w.mlp_down, [(partial_dn, hd)], "f32", shared, "postgate")
    dn = graph.buffer(n * hd * 4)
    comm.reduce_scatter(partial_dn, dn, n * hd, "f32")
    if defer:
        graph.release(mark, [x1, dn])
        return Residual(x1, dn)
    out = ops.add(graph, x1, dn, n * hd)
    graph.release(mark, [out])
    return out


def block_flops(cfg: BlockConfig, tokens: int) -> dict:
    """Multiply-add work of one block (2 FLOP per MAC): linears and attention (4 T^2 H D). A double block over the
    same tokens does the same work (each row goes through one stream's linears)."""
    hd, kvd = cfg.hidden, cfg.kv_heads * cfg.head_dim
    lin = 2 * tokens * (hd * hd * (2 + (1 if cfg.attn_gate else 0)) + 2 * hd * kvd
                        + hd * cfg.mlp * (3 if cfg.mlp_act == "swiglu" else 2))
    attn = 4 * tokens * tokens * cfg.heads * cfg.head_dim
    return {"linear": lin, "attention": attn, "total": lin + attn}
