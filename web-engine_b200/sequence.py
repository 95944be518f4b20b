"""Sequence parallelism of one image's step over the GPUs of a process group (one process per GPU).

The reference runs on one GPU. Here a step of one image can be split across N GPUs (the "step at 1/2/4/8 B200"
measurement): every rank keeps the model's weights (8.6 GB of fp8 for BASELINE config 4, well inside 180 GB of
HBM) and owns T/N consecutive rows of the token sequence. Linears, norms, RoPE and the residual stream run on the
rank's rows only. Attention needs every token, so q, k and v go through one all-to-all each (token shard, all
heads -> all tokens, H/N heads), each rank attends its heads, and the output comes back the same way:

    rows   [T/N, H, 128]  --we_head_groups-->  [N, T/N, H/N, 128]  --all_to_all-->  [T, H/N, 128]   (q, k, v)
    [T, H/N, 128]  --all_to_all-->  [N, T/N, H/N, 128]  --we_head_groups-->  [T/N, H, 128]           (o)

Per GPU and block that moves 4 x (N - 1)/N x T/N x H x 256 bytes: 12.4 MB at N = 8 for config 4, against about
100 MB for the tensor-parallel all-gather / reduce-scatter of the same block. The collectives are NCCL through
torch.distributed, on the torch stream the library's context uses.
"""
from __future__ import annotations

import ctypes as C

from . import _lib as L
from .graph import Graph, addr


class SequenceParallel:
    def __init__(self, group=None, device=None):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.device = device if device is not None else torch.device("cuda", torch.cuda.current_device())
        self._bufs: dict = {}

    def shard(self, tokens: int) -> tuple:
        """(first row, rows) of this rank: tokens split into equal consecutive shards."""
        if tokens % self.world:
            raise ValueError(f"{tokens} tokens do not split over {self.world} ranks")
        n = tokens // self.world
        return self.rank * n, n

    def buffer(self, key: str, nbytes: int):
        """A torch uint8 device buffer of at least nbytes, kept across blocks under `key`."""
        b = self._bufs.get(key)
        if b is None or b.numel() < nbytes:
            b = self.torch.empty(nbytes, dtype=self.torch.uint8, device=self.device)
            self._bufs[key] = b
        return b[:nbytes]

    def scatter_heads(self, graph: Graph, rows, local_tokens: int, heads: int, head_bytes: int, out_key: str):
        """rows [local_tokens, heads, head_bytes] of this rank -> [world * local_tokens, heads / world, head_bytes]
        (every token, this rank's heads); returns the torch buffer holding it."""
        if heads % self.world:
            raise ValueError(f"{heads} heads do not split over {self.world} ranks")
        gbytes = heads // self.world * head_bytes
        nbytes = local_tokens * heads * head_bytes
        send = self.buffer("send_" + out_key, nbytes)
        recv = self.buffer(out_key, nbytes)
        L.check(graph.ctx, L.lib().we_head_groups(graph.ctx, addr(rows), C.c_void_p(send.data_ptr()), local_tokens,
                                                  self.world, gbytes, 1))
        self.dist.all_to_all_single(recv, send, group=self.group)
        return recv

    def gather_heads(self, graph: Graph, heads_buf, local_tokens: int, heads: int, head_bytes: int, rows) -> None:
        """heads_buf (a torch buffer from `buffer`): [world * local_tokens, heads / world, head_bytes], every token
        with this rank's heads -> rows [local_tokens, heads, head_bytes] of this rank."""
        gbytes = heads // self.world * head_bytes
        nbytes = local_tokens * heads * head_bytes
        recv = self.buffer("gather_recv", nbytes)
        self.dist.all_to_all_single(recv, heads_buf[:nbytes], group=self.group)
        L.check(graph.ctx, L.lib().we_head_groups(graph.ctx, addr(rows), C.c_void_p(recv.data_ptr()), local_tokens,
                                                  self.world, gbytes, 0))

    def all_gather_rows(self, graph: Graph, local, local_bytes: int):
        """Every rank's `local_bytes` in rank order (a torch buffer of world * local_bytes)."""
        src = self.buffer("ag_src", local_bytes)
        graph.copy(local, 0, src.data_ptr(), 0, local_bytes)
        out = self.buffer("ag_out", local_bytes * self.world)
        self.dist.all_gather_into_tensor(out, src, group=self.group)
        return out
