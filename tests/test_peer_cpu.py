"""Host-side checks of the peer-memory exchange of sequence parallelism (web-engine_b200/sequence.py): the
we_peer_copy descriptors built for the head scatter, the head gather and the row all-gather, applied by a numpy
emulation of the kernel's copy rule to every rank's memory, give the all-to-all layouts the attention path
expects. No GPU."""
import numpy as np
import pytest

from conftest import load_package


def _apply(copies_per_rank, srcs, world, region_bytes):
    """The copy rule of we_peer_exchange: for each rank r, copy c, peer p and row i, chunk_bytes from
    srcs[r][c] at p * src_peer_stride + i * src_row_stride to region_p at dst_offset + r * dst_rank_stride +
    i * dst_row_stride. `src` fields are ignored (the emulation takes the bytes from srcs)."""
    regions = [np.zeros(region_bytes, np.uint8) for _ in range(world)]
    for r in range(world):
        for c, cp in enumerate(copies_per_rank[r]):
            src = srcs[r][c]
            n = cp["chunk_bytes"]
            for p in range(world):
                for i in range(cp["rows"]):
                    s0 = p * cp["src_peer_stride"] + i * cp["src_row_stride"]
                    d0 = cp["dst_offset"] + r * cp["dst_rank_stride"] + i * cp["dst_row_stride"]
                    assert d0 >= 0 and d0 + n <= region_bytes and s0 + n <= src.size
                    regions[p][d0:d0 + n] = src[s0:s0 + n]
    return regions


@pytest.mark.parametrize("world,heads,kv_heads", [(2, 4, 2), (4, 8, 4), (8, 8, 8)])
def test_scatter_then_gather_is_the_all_to_all(world, heads, kv_heads):
    seq = load_package().sequence
    t, hb = 3, 32  # tokens per rank, bytes per head
    rng = np.random.default_rng(world)
    q = [rng.integers(0, 256, t * heads * hb, dtype=np.uint8) for _ in range(world)]
    k = [rng.integers(0, 256, t * kv_heads * hb, dtype=np.uint8) for _ in range(world)]
    T, hl, kl = t * world, heads // world, kv_heads // world
    off_q, off_k = 0, T * hl * hb
    size = off_k + T * kl * hb
    copies = [[seq.scatter_copy(0, t, heads, hb, world, off_q), seq.scatter_copy(0, t, kv_heads, hb, world, off_k)]
              for _ in range(world)]
    regions = _apply(copies, [[q[r], k[r]] for r in range(world)], world, size)
    for me in range(world):
        # rank `me` holds every token (rank-major) with its heads [me hl, me hl + hl)
        want_q = np.concatenate([q[r].reshape(t, heads, hb)[:, me * hl:(me + 1) * hl] for r in range(world)])
        want_k = np.concatenate([k[r].reshape(t, kv_heads, hb)[:, me * kl:(me + 1) * kl] for r in range(world)])
        assert np.array_equal(regions[me][off_q:off_k].reshape(T, hl, hb), want_q)
        assert np.array_equal(regions[me][off_k:size].reshape(T, kl, hb), want_k)
    # identity attention: the gather brings every rank's own q rows back
    oh = [regions[me][off_q:off_k].copy() for me in range(world)]
    back = _apply([[seq.gather_copy(0, t, heads, hb, world, 0)] for _ in range(world)], [[oh[r]] for r in range(world)],
                  world, t * heads * hb)
    for me in range(world):
        assert np.array_equal(back[me], q[me])


def test_rows_copy_is_an_all_gather():
    seq = load_package().sequence
    world, nbytes = 4, 3 * 1024 + 512
    rng = np.random.default_rng(7)
    rows = [rng.integers(0, 256, nbytes, dtype=np.uint8) for _ in range(world)]
    cp = seq.rows_copy(0, nbytes)
    assert cp["chunk_bytes"] % 16 == 0 and nbytes % cp["chunk_bytes"] == 0 and cp["rows"] > 1
    regions = _apply([[cp] for _ in range(world)], [[rows[r]] for r in range(world)], world, world * nbytes)
    for me in range(world):
        assert np.array_equal(regions[me], np.concatenate(rows))
