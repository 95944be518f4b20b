"""GPU parity of attention (src/kernels/attention.ts:20-51) against the float64 oracle.

The f32 cases are the reference's own tests (tests/gpu/attention.test.ts: GQA shapes, query chunks, causal;
max abs error < 1e-5) and run on the CUDA-core kernel. The bf16 cases run the tcgen05 flash-attention kernel
(dim 128, no mask): ragged token counts, GQA groups, scores large enough to force the lazy rescaling, and
config 3's full size (4608 tokens x 24 heads) with oracle rows; tolerance cosine >= 0.9999 and max-abs-rel
< 1e-2 against float64 on the same bf16 inputs (P is rounded to bf16 for the second MMA).
"""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, lcg_floats, randn

pytestmark = pytest.mark.gpu


def run(we, graph, q, k, v, tokens, heads, kv_heads, dim, causal=False, dtype="f32", chunk=None):
    mark = graph.mark()
    try:
        conv = (lambda a: bf16(a)) if dtype == "bf16" else (lambda a: np.asarray(a, np.float32))
        qb, kb, vb = graph.buffer(conv(q)), graph.buffer(conv(k)), graph.buffer(conv(v))
        before = graph.stats["launches"]
        out = we.attention(graph, qb, kb, vb, tokens, heads, kv_heads, dim, causal=causal, chunk=chunk, dtype=dtype,
                           out_dtype="f32")
        launched = graph.stats["launches"] - before
        got = graph.read(out, tokens * heads * dim * 4, np.float32).copy()
        assert graph.device_error() == 0
        return got, launched
    finally:
        graph.release(mark)


@pytest.mark.parametrize("tokens,heads,kv_heads,dim", [(37, 4, 1, 128), (64, 8, 2, 128)])
def test_attention_matches_cpu_reference(we, graph, tokens, heads, kv_heads, dim):  # attention.test.ts:33-50
    r = lcg_floats(tokens * heads * dim + 2 * tokens * kv_heads * dim, 1, 2.0)
    q = r[: tokens * heads * dim]
    k = r[tokens * heads * dim: tokens * heads * dim + tokens * kv_heads * dim]
    v = r[tokens * heads * dim + tokens * kv_heads * dim:]
    got, _ = run(we, graph, q, k, v, tokens, heads, kv_heads, dim)
    assert np.max(np.abs(got - O.attention(q, k, v, tokens, heads, kv_heads, dim))) < 1e-5


def test_attention_in_query_chunks_is_the_same(we, graph):  # attention.test.ts:60-77
    tokens, heads, kv_heads, dim = 50, 2, 1, 16
    q, k, v = randn(tokens * heads * dim, 2), randn(tokens * dim, 3), randn(tokens * dim, 4)
    whole, _ = run(we, graph, q, k, v, tokens, heads, kv_heads, dim)
    chunked, _ = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, chunk=16)
    assert np.max(np.abs(chunked - whole)) < 1e-6
    assert np.max(np.abs(chunked - O.attention(q, k, v, tokens, heads, kv_heads, dim))) < 1e-5


def test_causal_attention(we, graph):  # attention.test.ts:80-96
    tokens, heads, kv_heads, dim = 19, 4, 1, 128
    q, k, v = randn(tokens * heads * dim, 5), randn(tokens * dim, 6), randn(tokens * dim, 7)
    got, _ = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, causal=True)
    assert np.max(np.abs(got - O.attention(q, k, v, tokens, heads, kv_heads, dim, causal=True))) < 1e-5


def test_attention_refuses_uneven_heads(we, graph):  # attention.test.ts:52-57
    b = graph.buffer(4)
    with pytest.raises(we._lib.WeError, match="multiple"):
        we.attention(graph, b, b, b, 1, 3, 2, 4)


def check(got, want):
    c = O.compare(got, want)
    rel = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    assert c["cosine"] >= 0.9999 and rel < 1e-2, (c, rel)


@pytest.mark.parametrize("tokens,heads,kv_heads", [(128, 2, 1), (200, 4, 2), (300, 3, 3), (1, 2, 1), (1024, 8, 2)])
def test_flash_attention_bf16(we, graph, tokens, heads, kv_heads):
    dim = 128
    q = bf16_round(randn(tokens * heads * dim, 11))
    k = bf16_round(randn(tokens * kv_heads * dim, 12))
    v = bf16_round(randn(tokens * kv_heads * dim, 13))
    got, launched = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, dtype="bf16")
    assert launched in (1, 2)  # the flash kernel (V read as stored, no transpose), + the combine if keys split
    check(got, O.attention(q, k, v, tokens, heads, kv_heads, dim))


def test_flash_attention_large_scores_rescale(we, graph):
    """Scores spread over hundreds of units: the running maximum grows by more than 2^8 many times."""
    tokens, heads, kv_heads, dim = 700, 2, 1, 128
    q = bf16_round(randn(tokens * heads * dim, 21, 4.0))
    k = bf16_round(randn(tokens * kv_heads * dim, 22, 4.0) * np.repeat(np.linspace(0.1, 2, tokens), dim)
                   .astype(np.float32))
    v = bf16_round(randn(tokens * kv_heads * dim, 23))
    got, _ = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, dtype="bf16")
    check(got, O.attention(q, k, v, tokens, heads, kv_heads, dim))


@pytest.mark.parametrize("tokens,heads,kv_heads,splits", [(1000, 2, 1, "3"), (600, 4, 2, "2"), (700, 1, 1, "5")])
def test_flash_attention_key_splits(we, graph, monkeypatch, tokens, heads, kv_heads, splits):
    """Keys split over CTAs (WE_FA_SPLITS forces it; the library splits by itself when a grid would not fill the
    GPU): unnormalised partial rows with their (max, sum), merged by the combine kernel."""
    monkeypatch.setenv("WE_FA_SPLITS", splits)
    dim = 128
    q = bf16_round(randn(tokens * heads * dim, 31))
    k = bf16_round(randn(tokens * kv_heads * dim, 32))
    v = bf16_round(randn(tokens * kv_heads * dim, 33))
    got, launched = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, dtype="bf16")
    assert launched == 2  # flash kernel + combine
    check(got, O.attention(q, k, v, tokens, heads, kv_heads, dim))


def test_flash_attention_splits_a_small_grid(we, graph):
    """4608 tokens x 3 heads (one rank's heads at 8-way sequence parallelism): 54 CTAs, so the keys split 3 ways."""
    tokens, heads, kv_heads, dim = 4608, 3, 3, 128
    rng = np.random.default_rng(9)
    q = bf16_round(rng.standard_normal(tokens * heads * dim, dtype=np.float32))
    k = bf16_round(rng.standard_normal(tokens * heads * dim, dtype=np.float32))
    v = bf16_round(rng.standard_normal(tokens * heads * dim, dtype=np.float32))
    got, launched = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, dtype="bf16")
    assert launched == 2
    rows = np.concatenate([np.arange(0, 16), rng.choice(tokens, 16, replace=False), np.arange(tokens - 16, tokens)])
    qq, kk, vv = (a.reshape(tokens, heads, dim).astype(np.float64) for a in (q, k, v))
    g3 = got.reshape(tokens, heads, dim)
    for h in range(heads):
        s = qq[rows, h] @ kk[:, h].T / np.sqrt(dim)
        p = np.exp(s - s.max(1, keepdims=True))
        check(g3[rows, h].ravel(), ((p / p.sum(1, keepdims=True)) @ vv[:, h]).ravel())


def test_flash_attention_config3_rows(we, graph):
    """Config 3's attention: 4608 tokens, 24 heads x 128, checked on 64 query rows of every head."""
    tokens, heads, kv_heads, dim = 4608, 24, 24, 128
    rng = np.random.default_rng(5)
    q = bf16_round(rng.standard_normal(tokens * heads * dim, dtype=np.float32))
    k = bf16_round(rng.standard_normal(tokens * heads * dim, dtype=np.float32))
    v = bf16_round(rng.standard_normal(tokens * heads * dim, dtype=np.float32))
    got, _ = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, dtype="bf16")
    rows = np.concatenate([np.arange(0, 16), rng.choice(tokens, 32, replace=False), np.arange(tokens - 16, tokens)])
    qq = q.reshape(tokens, heads, dim).astype(np.float64)
    kk = k.reshape(tokens, heads, dim).astype(np.float64)
    vv = v.reshape(tokens, heads, dim).astype(np.float64)
    g3 = got.reshape(tokens, heads, dim)
    for h in range(heads):
        s = qq[rows, h] @ kk[:, h].T / np.sqrt(dim)
        p = np.exp(s - s.max(1, keepdims=True))
        want = (p / p.sum(1, keepdims=True)) @ vv[:, h]
        check(g3[rows, h].ravel(), want.ravel())


def test_bf16_with_causal_runs_on_cuda_cores(we, graph):
    tokens, heads, kv_heads, dim = 40, 2, 1, 128
    q = bf16_round(randn(tokens * heads * dim, 31))
    k = bf16_round(randn(tokens * dim, 32))
    v = bf16_round(randn(tokens * dim, 33))
    got, launched = run(we, graph, q, k, v, tokens, heads, kv_heads, dim, causal=True, dtype="bf16")
    assert launched == 1
    assert np.max(np.abs(got - O.attention(q, k, v, tokens, heads, kv_heads, dim, causal=True))) < 1e-5
