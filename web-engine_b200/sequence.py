"""Sequence parallelism of one image's step over the GPUs of a process group (one process per GPU).

The reference runs on one GPU. Here a step of one image can be split across N GPUs (the "step at 1/2/4/8 B200"
measurement): every rank keeps the model's weights (8.6 GB of fp8 for BASELINE config 4, well inside 180 GB of
HBM) and owns T/N consecutive rows of the token sequence. Linears, norms, RoPE and the residual stream run on the
rank's rows only. Attention needs every token, so q, k and v go through one all-to-all each (token shard, all
heads -> all tokens, H/N heads), each rank attends its heads, and the output comes back the same way:

    rows   [T/N, H, 128]  --we_head_groups-->  [N, T/N, H/N, 128]  --all_to_all-->  [T, H/N, 128]   (q, k, v)
    [T, H/N, 128]  --all_to_all-->  [N, T/N, H/N, 128]  --we_head_groups-->  [T/N, H, 128]           (o)

Per GPU and block that moves 4 x (N - 1)/N x T/N x H x 256 bytes: 12.4 MB at N = 8 for config 4, against about
100 MB for the tensor-parallel all-gather / reduce-scatter of the same block.

Two ways to run the exchange:
  * peer (default): the library's peer-memory exchange (we_peer_exchange). Each rank's exchange region is opened
    by every other rank through CUDA IPC, and ONE kernel per exchange writes every (rank, token) chunk of q, k
    and v straight into the rank that attends those heads, over NVLink, then meets the others at a flag barrier
    in the same memory; the output comes back the same way. Three launches per block, no collective library on
    the data path, and the step can be captured in a CUDA graph. The regions alternate between even and odd
    blocks (a rank can never be two exchanges ahead of another).
  * nccl: we_head_groups to regroup the rows, then an NCCL all-to-all (we_all_to_all).
Both run over a comm.Comm (the library's NCCL communicator): the peer path uses it to pass the exchange regions'
handles, the nccl path for the all-to-all itself. No framework is involved.
"""
from __future__ import annotations

import ctypes as C

from . import _lib as L
from .graph import Buffer, Graph, addr


class PeerExchange:
    """This rank's exchange region in peer memory and every other rank's, opened once (we_peer_create / export /
    open; the handles travel through the communicator). exchange() runs one we_peer_exchange kernel."""

    def __init__(self, graph: Graph, nbytes: int, comm):
        self.graph = graph
        self.rank, self.world = comm.rank, comm.world
        self.nbytes = nbytes
        h = C.c_void_p()
        L.check(graph.ctx, L.lib().we_peer_create(graph.ctx, self.rank, self.world, nbytes, C.byref(h)))
        self.handle = h
        blob = (C.c_ubyte * L.PEER_HANDLE_BYTES)()
        L.check(graph.ctx, L.lib().we_peer_export(h, blob))
        blobs = comm.all_gather_bytes(bytes(blob))
        allb = (C.c_ubyte * (L.PEER_HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(blobs))
        L.check(graph.ctx, L.lib().we_peer_open(h, allb))
        self.region = L.lib().we_peer_region(h)

    def exchange(self, copies: list, timeout_ns: int = 0) -> None:
        """copies: dicts of we_peer_copy fields (src, rows, chunk_bytes, src_row_stride, src_peer_stride,
        dst_offset, dst_row_stride, dst_rank_stride)."""
        arr = (L.PeerCopy * len(copies))(*[L.PeerCopy(**c) for c in copies])
        L.check(self.graph.ctx, L.lib().we_peer_exchange(self.graph.ctx, self.handle, arr, len(copies), timeout_ns))

    def destroy(self) -> None:
        if self.handle is not None:
            L.lib().we_peer_destroy(self.handle)
            self.handle = None


def scatter_copy(src: int, t: int, heads: int, head_bytes: int, world: int, dst_offset: int) -> dict:
    """we_peer_copy of rows [t, heads, head_bytes] -> each rank p receives heads [p H/w, (p+1) H/w) of these rows
    at rows [rank t, rank t + t) of its [w t, H/w, head_bytes] block at dst_offset."""
    g = heads // world * head_bytes
    return dict(src=src, rows=t, chunk_bytes=g, src_row_stride=heads * head_bytes, src_peer_stride=g,
                dst_offset=dst_offset, dst_row_stride=g, dst_rank_stride=t * g)


def gather_copy(src: int, t: int, heads: int, head_bytes: int, world: int, dst_offset: int) -> dict:
    """we_peer_copy of this rank's heads over every token, [w t, H/w, head_bytes] -> rank p receives rows
    [p t, p t + t) as heads [rank H/w, ...) of its [t, H, head_bytes] block at dst_offset."""
    g = heads // world * head_bytes
    return dict(src=src, rows=t, chunk_bytes=g, src_row_stride=g, src_peer_stride=t * g, dst_offset=dst_offset,
                dst_row_stride=heads * head_bytes, dst_rank_stride=g)


def rows_copy(src: int, nbytes: int, dst_offset: int = 0) -> dict:
    """we_peer_copy of nbytes to every rank, at dst_offset + rank * nbytes (an all-gather), in chunks that keep
    many warps busy."""
    c = _chunk(nbytes)
    return dict(src=src, rows=nbytes // c, chunk_bytes=c, src_row_stride=c, src_peer_stride=0, dst_offset=dst_offset,
                dst_row_stride=c, dst_rank_stride=nbytes)


def _chunk(nbytes: int, limit: int = 4096) -> int:
    """The largest power-of-two chunk <= limit (and >= 16) that divides nbytes."""
    c = limit
    while c > 16 and nbytes % c:
        c //= 2
    return c


class SequenceParallel:
    """One image's rows split over the ranks of `comm` (a comm.Comm on the step's graph). peer: the peer-memory
    exchange kernel (default), else NCCL all-to-all. Buffers that live across blocks (the head blocks of the NCCL
    path and the attention output) are kept in a private library context, outside the step's mark / release
    scopes."""

    def __init__(self, comm, peer: bool = True, fused: bool = False):
        self.comm = comm
        self.rank, self.world = comm.rank, comm.world
        self.peer = peer
        # fused: the producers of q, k and v store them into the attending ranks' regions (head_targets /
        # finish_heads) instead of a copy kernel after them (exchange_heads). Measured on config 4 from a CUDA graph:
        # 45.3 ms fused against 44.7 ms with the copy kernel at 2 ranks, 20.5 against 19.45 ms at 8, so the copy
        # kernel is the default.
        self.fused = peer and fused
        self._pending = None
        self._store = Graph(comm.graph.device)  # persistent buffers only; no kernel runs on its stream
        self._bufs: dict = {}
        self._px: dict = {}  # PeerExchange per use ("heads", "rows"), grown collectively when a call needs more
        self._parity = 0
        self._rows_parity = 0

    def _exchange(self, graph: Graph, key: str, nbytes: int) -> PeerExchange:
        px = self._px.get(key)
        if px is None or px.nbytes < nbytes or px.graph is not graph:
            if px is not None:
                px.destroy()
            px = PeerExchange(graph, nbytes, self.comm)
            self._px[key] = px
        return px

    def destroy(self) -> None:
        """Frees the peer regions once every rank is done with them (a collective: every rank calls it)."""
        if self._px:
            self.comm.barrier()
        for px in self._px.values():
            px.destroy()
        self._px.clear()
        self._bufs.clear()
        self._store.destroy()

    def prepare(self, graph: Graph, local_tokens: int, heads: int, kv_heads: int, head_bytes: int) -> None:
        """Creates the exchange region and buffers that exchange_heads needs for this geometry now (a collective),
        so that it allocates nothing later: needed before capturing the blocks in a CUDA graph."""
        if not self.peer:
            raise ValueError("only the peer exchange can be captured in a CUDA graph (NCCL calls are not recorded)")
        t, w = local_tokens, self.world
        gq, gk = heads // w * head_bytes, kv_heads // w * head_bytes
        self._exchange(graph, "heads", 2 * (w * t * gq + 2 * w * t * gk + t * heads * head_bytes))
        self.buffer("o_heads", w * t * gq)

    def exchange_heads(self, graph: Graph, q, k, v, local_tokens: int, heads: int, kv_heads: int, head_bytes: int,
                       attend) -> int:
        """Peer path of one block's attention: q [t, heads], k / v [t, kv_heads] rows of this rank (head_bytes per
        head) go to the ranks that attend their heads; attend(qh, kh, vh, oh) runs this rank's heads over every
        token ([world * t, heads / world] each, oh a buffer it fills); the output comes back. Returns the device
        address of this rank's output rows [t, heads, head_bytes] (valid until the block after next)."""
        if heads % self.world or kv_heads % self.world:
            raise ValueError(f"{heads} / {kv_heads} heads do not split over {self.world} ranks")
        t, w = local_tokens, self.world
        T = t * w
        gq, gk = heads // w * head_bytes, kv_heads // w * head_bytes
        qb, kb, ob = T * gq, T * gk, t * heads * head_bytes
        per_set = qb + 2 * kb + ob
        px = self._exchange(graph, "heads", 2 * per_set)
        base = self._parity * per_set
        self._parity ^= 1
        off_q, off_k, off_v, off_o = base, base + qb, base + qb + kb, base + qb + 2 * kb

        px.exchange([scatter_copy(addr(q).value, t, heads, head_bytes, w, off_q),
                     scatter_copy(addr(k).value, t, kv_heads, head_bytes, w, off_k),
                     scatter_copy(addr(v).value, t, kv_heads, head_bytes, w, off_v)])
        oh = self.buffer("o_heads", qb)
        attend(px.region + off_q, px.region + off_k, px.region + off_v, oh)
        px.exchange([gather_copy(oh.ptr, t, heads, head_bytes, w, off_o)])
        return px.region + off_o

    def _head_sets(self, local_tokens: int, heads: int, kv_heads: int, head_bytes: int) -> tuple:
        """Byte sizes of one exchange set: q, k (= v) blocks of every token and this rank's heads, and the output."""
        t, w = local_tokens, self.world
        gq, gk = heads // w * head_bytes, kv_heads // w * head_bytes
        qb, kb, ob = t * w * gq, t * w * gk, t * heads * head_bytes
        return qb, kb, ob

    def head_targets(self, graph: Graph, local_tokens: int, heads: int, kv_heads: int, head_bytes: int) -> dict:
        """Fused path, first half of one block's attention exchange: the device addresses where the kernels that
        produce q, k and v store them directly (q / k norm + RoPE, the q/k/v GEMM's epilogue): for each, every
        rank's [world x local_tokens, heads / world, head_bytes] block in its region (this block's set of the two
        that blocks use in turn), with this rank's rows from row `row0`. finish_heads completes the exchange."""
        if heads % self.world or kv_heads % self.world:
            raise ValueError(f"{heads} / {kv_heads} heads do not split over {self.world} ranks")
        qb, kb, ob = self._head_sets(local_tokens, heads, kv_heads, head_bytes)
        per_set = qb + 2 * kb + ob
        px = self._exchange(graph, "heads", 2 * per_set)
        base = self._parity * per_set
        self._parity ^= 1
        offs = dict(q=base, k=base + qb, v=base + qb + kb, o=base + qb + 2 * kb)
        remote = [L.lib().we_peer_remote(px.handle, r) for r in range(self.world)]
        self._pending = (px, offs, qb)
        return {key: [r + offs[key] for r in remote] for key in ("q", "k", "v")} | {"row0": self.rank * local_tokens}

    def finish_heads(self, graph: Graph, local_tokens: int, heads: int, head_bytes: int, attend) -> int:
        """Fused path, second half: a flag barrier (the exchange kernel with no copies) after which every rank's
        stores into this rank's region are visible, attend(qh, kh, vh, oh) on them, and the output rows back (a
        copy exchange). Returns the device address of this rank's output rows [t, heads, head_bytes]."""
        px, offs, qb = self._pending
        self._pending = None
        px.exchange([])
        oh = self.buffer("o_heads", qb)
        attend(px.region + offs["q"], px.region + offs["k"], px.region + offs["v"], oh)
        px.exchange([gather_copy(oh.ptr, local_tokens, heads, head_bytes, self.world, offs["o"])])
        return px.region + offs["o"]

    def shard(self, tokens: int) -> tuple:
        """(first row, rows) of this rank: tokens split into equal consecutive shards."""
        if tokens % self.world:
            raise ValueError(f"{tokens} tokens do not split over {self.world} ranks")
        n = tokens // self.world
        return self.rank * n, n

    def buffer(self, key: str, nbytes: int) -> Buffer:
        """A device buffer of at least nbytes, kept across blocks under `key` (in the private context)."""
        b = self._bufs.get(key)
        if b is None or b.size < nbytes:
            if b is not None:
                self._store.free(b)
            b = self._store.buffer(nbytes)
            self._store.sync()  # its zero fill ran on the private stream: done before the step's stream uses it
            self._bufs[key] = b
        return b

    def scatter_heads(self, graph: Graph, rows, local_tokens: int, heads: int, head_bytes: int, out_key: str):
        """rows [local_tokens, heads, head_bytes] of this rank -> [world * local_tokens, heads / world, head_bytes]
        (every token, this rank's heads); returns the buffer holding it."""
        if heads % self.world:
            raise ValueError(f"{heads} heads do not split over {self.world} ranks")
        gbytes = heads // self.world * head_bytes
        nbytes = local_tokens * heads * head_bytes
        send = self.buffer("send_" + out_key, nbytes)
        recv = self.buffer(out_key, nbytes)
        L.check(graph.ctx, L.lib().we_head_groups(graph.ctx, addr(rows), C.c_void_p(send.ptr), local_tokens,
                                                  self.world, gbytes, 1))
        self.comm.all_to_all(send, recv, nbytes // self.world)
        return recv

    def gather_heads(self, graph: Graph, heads_buf, local_tokens: int, heads: int, head_bytes: int, rows) -> None:
        """heads_buf (a buffer from `buffer`): [world * local_tokens, heads / world, head_bytes], every token with
        this rank's heads -> rows [local_tokens, heads, head_bytes] of this rank."""
        gbytes = heads // self.world * head_bytes
        nbytes = local_tokens * heads * head_bytes
        recv = self.buffer("gather_recv", nbytes)
        self.comm.all_to_all(heads_buf, recv, nbytes // self.world)
        L.check(graph.ctx, L.lib().we_head_groups(graph.ctx, addr(rows), C.c_void_p(recv.ptr), local_tokens,
                                                  self.world, gbytes, 0))

    def all_gather_rows(self, graph: Graph, local, local_bytes: int):
        """Every rank's `local_bytes` in rank order: a device address (valid until the call after next) of
        world * local_bytes."""
        if self.peer:
            # two halves used in turn, like the head exchange: a rank may start the next call's copies into a
            # region that another rank still reads from this call's result
            px = self._exchange(graph, "rows", 2 * self.world * local_bytes)
            off = self._rows_parity * self.world * local_bytes
            self._rows_parity ^= 1
            px.exchange([rows_copy(addr(local).value, local_bytes, off)])
            return px.region + off
        out = self.buffer("ag_out", local_bytes * self.world)
        self.comm.all_gather(local, out, local_bytes)
        return out.ptr
