"""The denoising step around the blocks (src/model/transformer.ts:41-176) and the sampler (src/model/sampler.ts).

One step, as transformer.ts:134-176 lays it out:

    t, tvec = time(timestep)                 tmlp2(gelu(tmlp0(sincos(1000 t))))  and  tproj(gelu(t)) -> 6 x hidden
    txt     = txt_in(context)                [L, hidden], cached per image (it does not depend on the timestep)
    img     = first(patchify(latent))        [rows * cols, hidden]
    x       = [txt; img]                     [T, hidden] f32 residual stream, T = L + rows * cols
    x       = double blocks (text rows / image rows with their own weights, one attention), then single blocks
    v       = unpatchify(last((1 + t + last_scale) norm(x) + t + last_shift)[L:])

The reference's model is Krea 2 (single-stream blocks only, a text encoder in front); the layout here is the
Flux-style MMDiT of the benchmark configs (`double` two-stream blocks, then `single` blocks, a linear text
projection). Every op is the reference's: linear, norm, rotate, attention, the elementwise steps.

`dtype="f32"` runs the reference's f32 op semantics. `dtype="bf16"` is the B200 path: bf16 latent and context,
fp8 tcgen05 GEMMs on the exact e4m3 split, fused norm + split, q/k norm + RoPE, flash attention, fused epilogues;
the residual stream stays f32.
"""
from __future__ import annotations

import dataclasses
import functools
import math
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L
from . import kernels as K
from . import ops
from .block import BlockConfig, BlockWeights, Part, TPLayer, block_flops, buffers_of, joint_block
from .graph import Buffer, Graph, addr
from .stream import Streamer

LATENT_CHANNELS = 16
TIME_DIM = 256

# Config 3/4 block: 3072 hidden, 24 x 128 heads, 4x GELU MLP, no attention gate; RoPE axes 16/56/56, theta 1e4
FLUX_BLOCK = BlockConfig(hidden=3072, mlp=12288, heads=24, kv_heads=24, head_dim=128, eps=1e-5, mlp_act="gelu",
                         attn_gate=False)


@dataclass
class StepConfig:
    block: BlockConfig = field(default_factory=lambda: FLUX_BLOCK)
    double: int = 19
    single: int = 38
    channels: int = LATENT_CHANNELS
    ctx_dim: int = 3072
    time_dim: int = TIME_DIM
    axes: tuple = (16, 56, 56)
    theta: float = 1e4


@dataclass
class TransformerWeights:
    """Device weights of the whole model (TransformerWeights, transformer.ts:20-37, Flux-style layout)."""

    first: ops.Linear            # [hidden, 4 channels]
    tmlp0: ops.Linear            # [hidden, time_dim]
    tmlp2: ops.Linear            # [hidden, hidden]
    tproj: ops.Linear            # [6 hidden, hidden]
    txt_in: ops.Linear           # [hidden, ctx_dim]
    double: list                 # [(txt BlockWeights, img BlockWeights)]
    single: list                 # [BlockWeights]
    last_norm: object            # [hidden]
    last_scale: object           # [hidden]
    last_shift: object           # [hidden]
    last_linear: ops.Linear      # [4 channels, hidden]


def timestep_embedding(timestep: float, dim: int = TIME_DIM) -> np.ndarray:
    """[cos(1000 t f_i), sin(1000 t f_i)], f_i = 10000^(-i / (dim / 2)) (transformer.ts:41-51)."""
    half = dim // 2
    arg = 1000.0 * timestep * np.exp(-math.log(10000.0) * np.arange(half) / half)
    return np.concatenate([np.cos(arg), np.sin(arg)]).astype(np.float32)


def patch_grid(height: int, width: int) -> tuple:
    """Token grid of a latent: 2x2 patches, odd sizes padded up (transformer.ts:53)."""
    return (height + 1) // 2, (width + 1) // 2


def patchify(graph: Graph, latent, height: int, width: int, tokens, channels: int = LATENT_CHANNELS,
             latent_dtype: str = "f32", tokens_dtype: str = "f32") -> None:
    """latent [C, H, W] -> tokens [rows * cols, 4C] on the device (transformer.ts:59-69)."""
    L.check(graph.ctx, L.lib().we_patchify(graph.ctx, addr(latent), L.DTYPES[latent_dtype], channels, height, width,
                                           addr(tokens), L.DTYPES[tokens_dtype]))


def unpatchify(graph: Graph, tokens, height: int, width: int, latent, channels: int = LATENT_CHANNELS,
               tokens_dtype: str = "f32", latent_dtype: str = "f32") -> None:
    """tokens [rows * cols, 4C] -> latent [C, H, W], padding cropped (transformer.ts:72-82)."""
    L.check(graph.ctx, L.lib().we_unpatchify(graph.ctx, addr(tokens), L.DTYPES[tokens_dtype], channels, height, width,
                                             addr(latent), L.DTYPES[latent_dtype]))


@functools.lru_cache(maxsize=16)
def _tables(text_tokens: int, rows: int, cols: int, axes: tuple, theta: float):
    """RoPE cos/sin of a sequence geometry (ropeTables(positions(...)), transformer.ts:158); computed once per
    geometry on the host, uploaded each step through the library's staging ring."""
    cos, sin, pairs = K.rope_tables(K.positions(text_tokens, rows, cols), axes, theta)
    cos.setflags(write=False)
    sin.setflags(write=False)
    return cos, sin, pairs


def time(graph: Graph, w: TransformerWeights, timestep: float, time_dim: int = TIME_DIM):
    """t [hidden] and tvec [6 hidden] for one timestep (transformer.ts:85-90); M = 1 linears."""
    emb = graph.buffer(timestep_embedding(timestep, time_dim))
    t = ops.linear(graph, ops.gelu(graph, ops.linear(graph, emb, w.tmlp0, 1), w.tmlp0.n), w.tmlp2, 1)
    tvec = ops.linear(graph, ops.gelu(graph, t, w.tmlp2.n), w.tproj, 1)
    return t, tvec


def text(graph: Graph, w: TransformerWeights, context, tokens: int, dtype: str = "f32") -> Buffer:
    """The text rows of the sequence: txt_in(context) [tokens, hidden] f32 (the Flux-style text projection; the
    reference's Krea 2 text stack, transformer.ts:93-117, is a different model's front end)."""
    return ops.linear(graph, context, w.txt_in, tokens, x_dtype=dtype, y_dtype="f32")


@dataclass
class StepInputs:
    """One image's step inputs (Inputs, transformer.ts:124-132). latent [C, H, W] and context [L, ctx_dim] are
    device buffers of `dtype` elements; text_cache: txt rows from an earlier step of the same image."""

    latent: object
    height: int
    width: int
    timestep: float
    context: object
    text_tokens: int
    text_cache: object = None
    latent_dtype: str | None = None  # the latent's element type when it differs from the step's (f32 sampler state)


def _layers(w: TransformerWeights, images: int, T: int, Lt: int, image: int, r0: int, n: int) -> list:
    """The parts of every block: double blocks split each image's text and image rows, single blocks take all rows;
    clipped to this rank's rows [r0, r0 + n) of the stacked sequence."""
    R = images * T

    def clip(lo, hi, wt):
        a, b = max(lo, r0), min(hi, r0 + n)
        return [Part(a - r0, b - a, wt)] if b > a else []

    layers = [[p for i in range(images) for p in clip(i * T, i * T + Lt, tw) + clip(i * T + Lt, (i + 1) * T, iw)]
              for tw, iw in w.double]
    return layers + [clip(0, R, bw) for bw in w.single]


def _streamed_linears(w: BlockWeights) -> list:
    """The fp8 linears of a block that the bf16 path reads (q/k/v fused when fuse_qkv made them so)."""
    names = ["wqkv"] if w.wqkv is not None else ["wq", "wk", "wv"]
    names += ["wo", "mlp_up", "mlp_down"]
    names += [nm for nm in ("gate", "mlp_gate") if getattr(w, nm) is not None]
    return names


class StreamedBlocks:
    """The blocks' fp8 linear weights in pinned host memory, copied to HBM one layer (a block: both parts of a double
    block) at a time by a streamer (we_streamer: cudaMemcpyAsync on a side stream into `slots` device slots, the
    following layers prefetched while a block runs). This is loadTransformer's per-block upload (src/model/
    weights.ts:94-131) made per step, for models larger than HBM or a memory budget that keeps only a few blocks
    resident: per-channel scales, biases, norms and modulation tables (a few KB a block) stay resident.

    Built from a model whose weights are on the device (their bytes are read back once into host blobs); the device
    copies are the caller's to keep or free. transformer(..., streamed=...) then runs every block on its slot."""

    def __init__(self, graph: Graph, w: TransformerWeights, slots: int = 3, align: int = 1024):
        self.graph = graph
        self.layers = [list(pair) for pair in w.double] + [[bw] for bw in w.single]
        self.entries = []  # per layer: [(part index, linear name, byte offset)]
        blobs = []
        for ws in self.layers:
            entries, off = [], 0
            for wi, bw in enumerate(ws):
                for name in _streamed_linears(bw):
                    lin = getattr(bw, name)
                    if lin.dtype != "fp8":
                        raise ValueError("streaming takes the blocks' fp8 linears")
                    off = -(-off // align) * align
                    entries.append((wi, name, off))
                    off += lin.n * lin.k
            blob = np.empty(off, np.uint8)
            for wi, name, o in entries:
                lin = getattr(ws[wi], name)
                blob[o:o + lin.n * lin.k] = graph.read(lin.buffer, lin.n * lin.k)
            self.entries.append(entries)
            blobs.append(blob)
        self.host_bytes = sum(b.nbytes for b in blobs)
        self.streamer = Streamer(graph, blobs, slots=slots)

    def bind(self, i: int) -> dict:
        """Layer i's weights on the device: {id(original BlockWeights): a copy whose streamed linears point into the
        layer's slot}. Work queued after this call on the graph's stream sees the copied bytes."""
        base = self.streamer.acquire(i)
        out = {}
        for wi, bw in enumerate(self.layers[i]):
            repl = {}
            for wj, name, o in self.entries[i]:
                if wj == wi:
                    lin = getattr(bw, name)
                    repl[name] = dataclasses.replace(lin, buffer=base + o)
            out[id(bw)] = dataclasses.replace(bw, **repl)
        return out

    def release(self, i: int) -> None:
        """Layer i's work is queued: its slot may be refilled once that work has run."""
        self.streamer.release(i)

    @property
    def stats(self) -> dict:
        return self.streamer.stats

    def close(self) -> None:
        self.streamer.close()


class StepGraph:
    """The blocks of a step (all 57 for config 4), recorded once as a CUDA graph for one geometry and replayed
    each step: the host issues one launch instead of about 1000, so a step no longer depends on how fast Python
    issues its ops. It owns the blocks' input rows and timestep vector; a step copies its own into them."""

    def __init__(self, graph: Graph, w: TransformerWeights, cfg: StepConfig, height: int, width: int,
                 text_tokens: int, images: int = 1, dtype: str = "bf16", sp=None):
        """sp: a sequence.SequenceParallel (peer exchange) to record this rank's shard of one image's blocks; every
        rank of the group builds its StepGraph at the same point (the exchange regions are created first)."""
        bc = cfg.block
        rows, cols = patch_grid(height, width)
        image = rows * cols
        T = text_tokens + image
        R = images * T
        if sp is not None and (images != 1 or dtype != "bf16"):
            raise ValueError("sequence parallelism splits one image's rows on the bf16 path")
        r0, n = sp.shard(T) if sp is not None else (0, R)
        self.key = (height, width, text_tokens, images, dtype)
        self.sp = sp
        self.rows, self.hidden = n, bc.hidden
        cos, sin, pairs = _tables(text_tokens, rows, cols, tuple(cfg.axes), float(cfg.theta))
        self.x_in = graph.buffer(n * bc.hidden * 4)
        self.tvec = graph.buffer(6 * bc.hidden * 4)
        if sp is not None:
            self.cos, self.sin = graph.buffer(cos[r0 * pairs:(r0 + n) * pairs]), graph.buffer(sin[r0 * pairs:(r0 + n) * pairs])
            sp.prepare(graph, n, bc.heads, bc.kv_heads, bc.head_dim * 2)
        else:
            self.cos, self.sin = graph.buffer(np.tile(cos, images)), graph.buffer(np.tile(sin, images))
        rope = ops.Rope(self.cos, self.sin, pairs, n)
        with graph.capture() as cap:
            x = self.x_in
            layers = _layers(w, images, T, text_tokens, image, r0, n)
            for i, parts in enumerate(layers):
                bm = graph.mark()
                nxt = joint_block(graph, parts, bc, x, self.tvec, rope, dtype, images=images, sp=sp,
                                  defer=i + 1 < len(layers))
                graph.release(bm, buffers_of(nxt))
                if x is not self.x_in:
                    for b in buffers_of(x):
                        graph.free(b)
                x = nxt
        self.captured, self.out = cap, x

    def run(self, graph: Graph, x, tvec) -> Buffer:
        """The blocks on x [rows, hidden] f32 with tvec [6 hidden]: a new result in self.out (graph-owned)."""
        graph.copy(x, 0, self.x_in, 0, self.rows * self.hidden * 4)
        graph.copy(tvec, 0, self.tvec, 0, 6 * self.hidden * 4)
        self.captured.launch()
        return self.out

    def destroy(self) -> None:
        self.captured.destroy()


def transformer(graph: Graph, w: TransformerWeights, cfg: StepConfig, inp, dtype: str = "f32", velocity=None,
                on_block=None, sp=None, captured: StepGraph | None = None,
                streamed: StreamedBlocks | None = None, tp=None) -> tuple:
    """One denoising step (transformer.ts:134-176) of one image (`inp` a StepInputs) or of a batch of images (a list
    of StepInputs with the same geometry and timestep). The batch runs as one token stream: every linear is one
    GEMM over all images' rows, attention runs per image.

    Returns the predicted velocity [C, H, W] f32 (a new buffer, or written into `velocity`) and the txt rows for
    the next step's text_cache; for a batch, lists of both.

    sp: a sequence.SequenceParallel to split one image's rows over the ranks of its group (bf16 path): each rank
    runs the blocks on T / world consecutive rows, attention exchanges heads by all-to-all, and every rank gets the
    whole velocity.

    captured: a StepGraph of this geometry; the blocks then run as its replay (on_block is not called).

    streamed: a StreamedBlocks of w: every block's fp8 linears are copied from pinned host memory into a device slot
    just ahead of the block (eager path only).

    tp: a parallel.TPGroup to split one image's step over the ranks of its communicator by tensor parallelism (bf16
    path, eager): w is this rank's sharded model (parallel.shard_model); each rank holds T / world rows of the
    residual stream, and every block gathers the split activations, runs this rank's heads and MLP columns over all
    rows and reduce-scatters its K-slice partial sums back to the rows' owners. Every rank gets the whole velocity."""
    batch = list(inp) if isinstance(inp, (list, tuple)) else [inp]
    b0 = batch[0]
    if any((b.height, b.width, b.text_tokens, b.timestep) != (b0.height, b0.width, b0.text_tokens, b0.timestep)
           for b in batch):
        raise ValueError("the images of a batch need the same size, text length and timestep")
    bc = cfg.block
    hid, ch, B = bc.hidden, cfg.channels, len(batch)
    rows, cols = patch_grid(b0.height, b0.width)
    image, Lt = rows * cols, b0.text_tokens
    T = Lt + image
    R = B * T
    cos, sin, pairs = _tables(Lt, rows, cols, tuple(cfg.axes), float(cfg.theta))
    if sp is not None and (B != 1 or dtype != "bf16"):
        raise ValueError("sequence parallelism runs one image on the bf16 path")
    if tp is not None and (B != 1 or dtype != "bf16" or sp is not None or captured is not None or streamed is not None):
        raise ValueError("tensor parallelism runs one image on the bf16 path, eagerly")
    group = sp if sp is not None else tp
    r0, n = group.shard(T) if group is not None else (0, R)  # this rank's rows
    outs = velocity if isinstance(velocity, (list, tuple)) else [velocity] * B if velocity is not None else [None] * B
    mark = graph.mark()
    t, tvec = time(graph, w, b0.timestep, cfg.time_dim)
    x = graph.buffer(R * hid * 4)
    es = 2 if dtype == "bf16" else 4
    tok = graph.buffer(B * image * 4 * ch * es)
    txts = []
    for i, ib in enumerate(batch):
        txt = ib.text_cache if ib.text_cache is not None else text(graph, w, ib.context, Lt, dtype)
        txts.append(txt)
        graph.copy(txt, 0, x, i * T * hid * 4, Lt * hid * 4)
        patchify(graph, ib.latent, ib.height, ib.width, addr(tok).value + i * image * 4 * ch * es, ch,
                 ib.latent_dtype or dtype, dtype)
    img = ops.linear(graph, tok, w.first, B * image, x_dtype=dtype, y_dtype="f32")
    for i in range(B):
        graph.copy(img, i * image * hid * 4, x, (i * T + Lt) * hid * 4, image * hid * 4)
    if group is not None:  # keep this rank's rows
        xs = graph.buffer(n * hid * 4)
        graph.copy(x, r0 * hid * 4, xs, 0, n * hid * 4)
        graph.free(x)
        x = xs
        rope = ops.Rope(graph.buffer(cos[r0 * pairs:(r0 + n) * pairs]), graph.buffer(sin[r0 * pairs:(r0 + n) * pairs]),
                        pairs, n)
    elif captured is None:  # (a captured step holds its own tables)
        rope = ops.Rope(graph.buffer(np.tile(cos, B)), graph.buffer(np.tile(sin, B)), pairs, R)

    if captured is not None:
        if captured.key != (b0.height, b0.width, Lt, B, dtype) or captured.sp is not sp:
            raise ValueError("the captured step is for another geometry, batch, dtype or sequence-parallel group")
        x = captured.run(graph, x, tvec)  # graph-owned; the last layer reads it
    else:
        if streamed is not None and captured is not None:
            raise ValueError("a streamed step runs eagerly")
        layers = _layers(w, B, T, Lt, image, r0, n)
        if tp is not None:  # every layer's parts over all T rows, and the tables of all rows, for the gathered GEMMs
            layers_all = _layers(w, B, T, Lt, image, 0, T)
            rope_all = ops.Rope(graph.buffer(cos), graph.buffer(sin), pairs, T)
        for i, parts in enumerate(layers):
            if streamed is not None:  # this block's linears from its slot (the same BlockWeights -> the same copy)
                bound = streamed.bind(i)
                parts = [Part(p.row0, p.rows, bound[id(p.w)]) for p in parts]
            bm = graph.mark()
            tpl = TPLayer(tp.comm, layers_all[i], rope_all) if tp is not None else None
            # between blocks the output stays a Residual: the next block's first norm pass adds it
            nxt = joint_block(graph, parts, bc, x, tvec, rope, dtype, images=B, sp=sp, defer=i + 1 < len(layers),
                              tp=tpl)
            if streamed is not None:
                streamed.release(i)
            graph.release(bm, buffers_of(nxt))
            for b in buffers_of(x):
                graph.free(b)
            x = nxt
            if on_block:
                on_block(i)
    scale = ops.add(graph, t, w.last_scale, hid)
    shift = ops.add(graph, t, w.last_shift, hid)
    if dtype == "bf16":
        split = (graph.buffer(n * hid), graph.buffer(n * hid), graph.buffer(n * 4))
        K.norm_split(graph, x, w.last_norm, n, hid, *split, scale=scale, shift=shift, eps=bc.eps)
        last = graph.buffer(n * 4 * ch * 4)
        K.gemm_fp8(graph, *split, w.last_linear.buffer, last, n, w.last_linear.n, w.last_linear.k,
                   w.last_linear.scale, chan_scale=w.last_linear.chan_scale, bias=w.last_linear.bias, y_dtype="f32")
        if sp is not None:  # every rank's rows of the last linear, in order
            last = sp.all_gather_rows(graph, last, n * 4 * ch * 4)
        elif tp is not None:
            gathered = graph.buffer(R * 4 * ch * 4)
            tp.comm.all_gather(last, gathered, n * 4 * ch * 4)
            last = gathered
    else:
        h = ops.norm(graph, x, w.last_norm, R, hid, ops.Mod(scale, shift), bc.eps)
        last = ops.linear(graph, h, w.last_linear, R)
    vel = []
    for i in range(B):
        out = outs[i] if outs[i] is not None else graph.buffer(ch * b0.height * b0.width * 4)
        unpatchify(graph, addr(last).value + (i * T + Lt) * 4 * ch * 4, b0.height, b0.width, out, ch, "f32", "f32")
        vel.append(out)
    keep = [b for b in vel + txts if isinstance(b, Buffer)]
    graph.release(mark, keep)
    if isinstance(inp, (list, tuple)):
        return vel, txts
    return vel[0], txts[0]


def step_flops(cfg: StepConfig, text_tokens: int, image_tokens: int) -> dict:
    """FLOPs of one step: the blocks (linears + attention) plus the first, text and last linears."""
    T = text_tokens + image_tokens
    b = block_flops(cfg.block, T)
    n = cfg.double + cfg.single
    hid = cfg.block.hidden
    edge = 2 * (image_tokens * 4 * cfg.channels * hid + text_tokens * cfg.ctx_dim * hid + T * hid * 4 * cfg.channels)
    return {"linear": n * b["linear"] + edge, "attention": n * b["attention"], "total": n * b["total"] + edge}


# ---------------- sampler (src/model/sampler.ts) ----------------
TURBO = {"steps": 8, "mu": 1.15}


def sigmas(steps: int = TURBO["steps"], mu: float = TURBO["mu"]) -> list:
    """linspace(1, 1/steps, steps) under the time shift e^mu / (e^mu + 1/s - 1), then 0 (sampler.ts:9-19)."""
    raw = [1 - i * (1 - 1 / steps) / ((steps - 1) or 1) for i in range(steps)]
    return [math.exp(mu) / (math.exp(mu) + (1 / s - 1)) for s in raw] + [0.0]


def euler_step(graph: Graph, x, velocity, sigma: float, nxt: float, n: int, out=None) -> Buffer:
    """x + (sigma_next - sigma) v on the device (eulerStep, sampler.ts:22-24), f32."""
    g = graph.buffer(np.array([nxt - sigma], np.float32))
    if out is None:
        out = ops.gated_add(graph, x, velocity, g, n, 1)
    else:
        L.check(graph.ctx, L.lib().we_elementwise(graph.ctx, L.EW["gated_add"], addr(x), addr(velocity), addr(g), n, 1,
                                                  L.DTYPES["f32"], addr(out), L.DTYPES["f32"]))
    graph.free(g)  # back to the pool: a later user of it is queued after this step
    return out


def gaussian(n: int, seed: int) -> np.ndarray:
    """Seeded standard normals: Box-Muller on a 32-bit LCG, u = (s + 0.5) / 2^32 (gaussian, sampler.ts:27-38)."""
    s = (seed & 0xFFFFFFFF) or 1
    m = (n + 1) // 2
    draws = np.empty(2 * m, dtype=np.uint64)
    for i in range(2 * m):  # the LCG is sequential; the transcendental part below is vectorised
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        draws[i] = s
    u = (draws.astype(np.float64) + 0.5) / 2.0 ** 32
    r, a = np.sqrt(-2.0 * np.log(u[0::2])), 2.0 * np.pi * u[1::2]
    out = np.empty(2 * m, dtype=np.float32)
    out[0::2], out[1::2] = r * np.cos(a), r * np.sin(a)
    return out[:n]


def sample(graph: Graph, w: TransformerWeights, cfg: StepConfig, noise: list, contexts: list, height: int, width: int,
           text_tokens: int, steps: int = TURBO["steps"], mu: float = TURBO["mu"], dtype: str = "bf16",
           on_step=None, streamed: StreamedBlocks | None = None) -> list:
    """Flow-matching Euler sampling of a batch of images (the loop of src/pipeline/generate.ts:94-105): the text
    rows are computed once per image, each step feeds timestep = sigma_i, then x += (sigma_{i+1} - sigma_i) v.
    noise: f32 latents [C, H, W] on the device (one per image); contexts: [text_tokens, ctx_dim] of `dtype`.
    Returns new f32 latent buffers."""
    sig = sigmas(steps, mu)
    n = cfg.channels * height * width
    xs, caches = list(noise), [None] * len(noise)
    for i in range(steps):
        inputs = [StepInputs(xs[b], height, width, sig[i], contexts[b], text_tokens, caches[b], latent_dtype="f32")
                  for b in range(len(xs))]
        vel, caches = transformer(graph, w, cfg, inputs, dtype, streamed=streamed)
        nxt = [euler_step(graph, xs[b], vel[b], sig[i], sig[i + 1], n) for b in range(len(xs))]
        for v in vel:
            graph.free(v)
        if i > 0:
            for x in xs:
                graph.free(x)
        xs = nxt
        if on_step:
            on_step(i)
    return xs
