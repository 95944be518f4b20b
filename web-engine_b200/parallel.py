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
