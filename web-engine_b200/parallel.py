"""Multi-GPU execution of the linear layers: tensor-parallel shards and data-parallel replicas.

One process per GPU; the collectives run on a communicator with comm.Comm's interface: the library's NCCL
communicator over NVLink/NVSwitch on B200 (we_all_gather / we_reduce_scatter through the C ABI), or, in the CPU
tests of the host logic, an adapter over gloo. The compute of every shard is the single-GPU operator
(``ops.linear``), so each rank runs the same kernels as one GPU does.

Tensor parallelism follows the Megatron + sequence-parallel layout of a DiT block (each block has four
collectives):
  * column-parallel (QKV, attention gate, MLP gate/up): W split along N. The token-sharded input
    [T/world, K] is all-gathered to [T, K]; each rank computes its N/world output columns (its heads).
  * row-parallel (attention out, MLP down): W split along K. Each rank multiplies its K/world slice
    of the activations; the f32 partial outputs [T, N] are reduce-scattered over tokens to [T/world, N].
Data parallelism runs one image batch per GPU with no collective on the data path.

The weight sharding keeps the on-disk formats: an fp8 weight's per-channel scales split with its rows;
an int4 group-64 weight splits along K only at group boundaries.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass
class Shard:
    """One rank's slice of a linear layer's weights (host arrays, before upload)."""

    weight: np.ndarray          # fp8 bytes [n, k] / bf16 bits [n, k] / int4 packed [n, k/2]
    dtype: str                  # "fp8" | "bf16" | "int4"
    n: int
    k: int
    scale: float = 1.0
    chan_scale: np.ndarray | None = None   # [n]
    group_scale: np.ndarray | None = None  # int4: f16 bits [n, k/64]
    bias: np.ndarray | None = None         # [n] (column-parallel only; row-parallel adds it after the reduction)


def split_range(total: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """[begin, end) of rank's part of `total`, in whole multiples of `align` (the last rank takes the rest)."""
    if total % align:
        raise ValueError(f"{total} is not a multiple of {align}")
    units = total // align
    per = -(-units // world)
    b = min(units, rank * per) * align
    e = min(units, (rank + 1) * per) * align
    return b, e


def shard_column(weight: np.ndarray, dtype: str, n: int, k: int, world: int, rank: int, *, scale: float = 1.0,
                 chan_scale=None, group_scale=None, bias=None, align: int = 1) -> Shard:
    """Rows (output channels) [b, e) of W [n, k]: the column-parallel shard."""
    b, e = split_range(n, world, rank, align)
    w = weight.reshape(n, -1)[b:e].copy()
    return Shard(w.ravel(), dtype, e - b, k, scale,
                 None if chan_scale is None else np.asarray(chan_scale)[b:e].copy(),
                 None if group_scale is None else np.asarray(group_scale).reshape(n, -1)[b:e].ravel().copy(),
                 None if bias is None else np.asarray(bias)[b:e].copy())


def shard_row(weight: np.ndarray, dtype: str, n: int, k: int, world: int, rank: int, *, scale: float = 1.0,
              chan_scale=None, group_scale=None) -> Shard:
    """Columns (input features) [b, e) of W [n, k]: the row-parallel shard. int4 splits at group (64) boundaries,
    fp8 at 16 values (the tensor-core kernel's row alignment)."""
    align = 64 if dtype == "int4" else 16
    b, e = split_range(k, world, rank, align)
    w2 = weight.reshape(n, -1)
    if dtype == "int4":
        w = w2[:, b // 2:e // 2]
        gs = None if group_scale is None else np.asarray(group_scale).reshape(n, k // 64)[:, b // 64:e // 64]
    else:
        w = w2[:, b:e]
        gs = None
    return Shard(np.ascontiguousarray(w).ravel(), dtype, n, e - b, scale,
                 None if chan_scale is None else np.asarray(chan_scale).copy(),
                 None if gs is None else np.ascontiguousarray(gs).ravel())


class TensorParallel:
    """The collective steps of a TP linear pair on a communicator (comm.Comm on GPUs).

    comm: all_gather(src, dst, nbytes) and reduce_scatter(src, dst, count, dtype) on buffers, rank and world;
    alloc(nbytes): a new buffer (graph.buffer on a GPU). matmul(x, shard, m) -> y is the single-device linear
    (``ops.linear`` on a GPU; the CPU tests pass the oracle); add_bias(y, bias, rows, n) -> y adds a full-width
    bias once after a reduction."""

    def __init__(self, comm, alloc):
        self.comm, self.alloc = comm, alloc
        self.world, self.rank = comm.world, comm.rank

    def all_gather_tokens(self, x_local, rows: int, row_bytes: int):
        """[rows, row_bytes] per rank -> [world * rows, row_bytes] on every rank (equal shards, rank order)."""
        out = self.alloc(self.world * rows * row_bytes)
        self.comm.all_gather(x_local, out, rows * row_bytes)
        return out

    def reduce_scatter_tokens(self, partial, rows: int, n: int, dtype: str = "f32"):
        """[rows, n] partial sums per rank -> this rank's [rows / world, n] of their sum."""
        if rows % self.world:
            raise ValueError(f"{rows} tokens do not split over {self.world} ranks")
        esz = 4 if dtype == "f32" else 2
        out = self.alloc(rows // self.world * n * esz)
        self.comm.reduce_scatter(partial, out, rows // self.world * n, dtype)
        return out

    def column_linear(self, matmul, x_local, rows: int, row_bytes: int, shard: Shard):
        """Column-parallel: gather the token shards ([rows, row_bytes] here), multiply by this rank's output
        channels."""
        x = self.all_gather_tokens(x_local, rows, row_bytes)
        return matmul(x, shard, self.world * rows)

    def row_linear(self, matmul, x_cols, rows: int, shard: Shard, bias=None, add_bias=None):
        """Row-parallel: this rank's K slice of the activations ([rows, shard.k]) times its K slice of W, summed
        over ranks and scattered over tokens (f32 partials). `bias` (full [N]) is added once, after the
        reduction."""
        partial = matmul(x_cols, shard, rows)
        y = self.reduce_scatter_tokens(partial, rows, shard.n)
        if bias is not None:
            y = add_bias(y, bias, rows // self.world, shard.n)
        return y


# ---------------- the tensor-parallel step: this rank's shards of a model's blocks ----------------
def _addr(b) -> int:
    from .graph import addr

    return addr(b).value


def shard_rows(graph, lin, r0: int, r1: int, keep_bias: bool = True):
    """Output channels [r0, r1) of a device fp8 / bf16 Linear (column-parallel shard), as new graph buffers."""
    from .ops import Linear

    es = 2 if lin.dtype == "bf16" else 1
    if lin.dtype not in ("fp8", "bf16"):
        raise ValueError("tensor-parallel shards take fp8 or bf16 weights")
    n = r1 - r0
    buf = graph.buffer(n * lin.k * es)
    graph.copy(lin.buffer, r0 * lin.k * es, buf, 0, n * lin.k * es)
    cs = bias = None
    if lin.chan_scale is not None:
        cs = graph.buffer(n * 4)
        graph.copy(lin.chan_scale, r0 * 4, cs, 0, n * 4)
    if lin.bias is not None and keep_bias:
        bias = graph.buffer(n * 4)
        graph.copy(lin.bias, r0 * 4, bias, 0, n * 4)
    return Linear(buf, lin.dtype, lin.scale, n, lin.k, bias=bias, chan_scale=cs)


def shard_cols(graph, lin, c0: int, c1: int, keep_bias: bool):
    """Input features [c0, c1) of a device fp8 / bf16 Linear (row-parallel shard: a strided copy of every row's K
    slice). The per-channel scale is the whole layer's (it multiplies each output channel, so the sum of the ranks'
    scaled partials is the scaled sum); the bias is kept by one rank only, so the reduction adds it once."""
    from .ops import Linear

    es = 2 if lin.dtype == "bf16" else 1
    if lin.dtype not in ("fp8", "bf16"):
        raise ValueError("tensor-parallel shards take fp8 or bf16 weights")
    kk = c1 - c0
    buf = graph.buffer(lin.n * kk * es)
    graph.copy_2d(_addr(lin.buffer) + c0 * es, lin.k * es, buf, kk * es, kk * es, lin.n)
    return Linear(buf, lin.dtype, lin.scale, lin.n, kk, bias=lin.bias if keep_bias else None,
                  chan_scale=lin.chan_scale)


def shard_block(graph, w, cfg, world: int, rank: int):
    """This rank's shard of a block's weights (block.BlockWeights) for block._joint_bf16_tp: q / k / v (fused when
    the block is), the attention gate and MLP gate / up split along their output channels (this rank's heads and
    MLP columns), wo and MLP down along K; norms and the modulation table are shared. Made once, outside any
    mark / release scope (new graph buffers)."""
    import dataclasses

    from .block import fuse_qkv

    if cfg.heads % world or cfg.kv_heads % world or cfg.mlp % world:
        raise ValueError(f"heads, kv heads and MLP width must split over {world} ranks")
    hd = cfg.head_dim
    hq, hk, ml = cfg.heads // world * hd, cfg.kv_heads // world * hd, cfg.mlp // world
    q0, k0, m0 = rank * hq, rank * hk, rank * ml
    first = rank == 0
    out = dict(wq=shard_rows(graph, w.wq, q0, q0 + hq), wk=shard_rows(graph, w.wk, k0, k0 + hk),
               wv=shard_rows(graph, w.wv, k0, k0 + hk), wo=shard_cols(graph, w.wo, q0, q0 + hq, first),
               mlp_up=shard_rows(graph, w.mlp_up, m0, m0 + ml), mlp_down=shard_cols(graph, w.mlp_down, m0, m0 + ml, first),
               gate=shard_rows(graph, w.gate, q0, q0 + hq) if w.gate is not None else None,
               mlp_gate=shard_rows(graph, w.mlp_gate, m0, m0 + ml) if w.mlp_gate is not None else None, wqkv=None)
    local = dataclasses.replace(w, **out)
    return fuse_qkv(graph, local) if w.wqkv is not None else local


def shard_model(graph, model, cfg, world: int, rank: int):
    """This rank's tensor-parallel model (transformer.TransformerWeights): every block sharded (shard_block), the
    edge linears (time MLP, text and latent projections, last layer) and the last norm shared as they are."""
    import dataclasses

    bc = cfg.block
    double = [(shard_block(graph, t, bc, world, rank), shard_block(graph, i, bc, world, rank)) for t, i in model.double]
    single = [shard_block(graph, b, bc, world, rank) for b in model.single]
    return dataclasses.replace(model, double=double, single=single)


class TPGroup:
    """A tensor-parallel group on a communicator (comm.Comm): transformer(..., tp=TPGroup(comm)) runs one image's
    step with every rank holding T / world rows of the residual stream and its shard of every block's linears."""

    def __init__(self, comm):
        self.comm = comm
        self.rank, self.world = comm.rank, comm.world

    def shard(self, tokens: int) -> tuple:
        """(first row, rows) of this rank: tokens split into equal consecutive shards."""
        if tokens % self.world:
            raise ValueError(f"{tokens} tokens do not split over {self.world} ranks")
        n = tokens // self.world
        return self.rank * n, n
