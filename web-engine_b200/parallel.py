"""Multi-GPU execution of the linear layers: tensor-parallel shards and data-parallel replicas.

One process per GPU; torch.distributed (NCCL over NVLink/NVSwitch on B200, gloo on CPU for the
host-logic tests) carries the collectives. The compute of every shard is the single-GPU operator
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
    """The collective steps of a TP linear pair on top of a torch.distributed process group.

    `matmul(x, shard, m) -> y` is the single-device linear (``ops.linear`` on a GPU; the tests pass
    the CPU oracle). Activations are torch tensors on the rank's device."""

    def __init__(self, group=None):
        import torch.distributed as dist

        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def all_gather_tokens(self, x_local):
        """[T/world, K] per rank -> [T, K] on every rank (equal shards)."""
        import torch

        out = torch.empty((self.world * x_local.shape[0],) + tuple(x_local.shape[1:]), dtype=x_local.dtype,
                          device=x_local.device)
        self.dist.all_gather_into_tensor(out, x_local.contiguous(), group=self.group)
        return out

    def reduce_scatter_tokens(self, partial):
        """[T, N] partial sums per rank -> this rank's [T/world, N] of the sum."""
        import torch

        t = partial.shape[0]
        if t % self.world:
            raise ValueError(f"{t} tokens do not split over {self.world} ranks")
        out = torch.empty((t // self.world,) + tuple(partial.shape[1:]), dtype=partial.dtype, device=partial.device)
        self.dist.reduce_scatter_tensor(out, partial.contiguous(), group=self.group)
        return out

    def column_linear(self, matmul, x_local, shard: Shard):
        """Column-parallel: gather the token shards, multiply by this rank's output channels."""
        x = self.all_gather_tokens(x_local)
        return matmul(x, shard, x.shape[0])

    def row_linear(self, matmul, x_cols, shard: Shard, bias=None):
        """Row-parallel: this rank's K slice of the activations times its K slice of W, summed over ranks
        and scattered over tokens. `bias` (full [N]) is added once, after the reduction."""
        partial = matmul(x_cols, shard, x_cols.shape[0])
        y = self.reduce_scatter_tokens(partial)
        if bias is not None:
            y = y + bias
        return y


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest `value` over all ranks (timings are reported as the max over ranks)."""
    import torch
    import torch.distributed as dist

    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
