"""The index math of the sequence-parallel exchange, no GPU: we_head_groups' layout (restated from its kernel:
word (t, g, v) of [tokens, groups, group words] <-> word (g, t, v) of [groups, tokens, group words]) followed by
all-to-all's chunk semantics gives every rank all tokens of its heads, and the reverse path gives back its rows."""
import numpy as np
import pytest


def to_groups(rows, groups):
    t, h, d = rows.shape
    return rows.reshape(t, groups, h // groups, d).transpose(1, 0, 2, 3).copy()  # [groups, t, h/groups, d]


def from_groups(grouped):
    g, t, hg, d = grouped.shape
    return grouped.transpose(1, 0, 2, 3).reshape(t, g * hg, d)


def all_to_all(sends):
    """sends[r][s] is what rank r sends to rank s; rank s receives [sends[0][s], sends[1][s], ...]."""
    world = len(sends)
    return [np.stack([sends[r][s] for r in range(world)]) for s in range(world)]


@pytest.mark.parametrize("world,tokens,heads", [(2, 80, 4), (4, 96, 8), (8, 4608, 24)])
def test_exchange_gives_each_rank_all_tokens_of_its_heads(world, tokens, heads):
    d = 3
    rng = np.random.default_rng(world)
    q = rng.standard_normal((tokens, heads, d))
    n, hg = tokens // world, heads // world
    shards = [q[r * n:(r + 1) * n] for r in range(world)]
    recv = all_to_all([to_groups(s, world) for s in shards])
    for r in range(world):
        assert np.array_equal(recv[r].reshape(tokens, hg, d), q[:, r * hg:(r + 1) * hg])
    # back: each rank's [tokens, hg, d] output -> chunks of n rows -> its row shard with every head
    outs = [recv[r].reshape(tokens, hg, d) * 2 for r in range(world)]
    back = all_to_all([o.reshape(world, n, hg, d) for o in outs])
    for r in range(world):
        assert np.array_equal(from_groups(back[r]), 2 * shards[r])
