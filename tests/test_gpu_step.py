"""GPU parity of the step driver (src/model/transformer.ts:41-176, src/model/sampler.ts).

- patchify / unpatchify on the device: bit-exact against the oracle on the reference test's shapes (even, odd
  and the 128x128 latent of a 1024x1024 image), f32 and bf16.
- the double-stream block (two parts, one attention) against the float64 joint-block restatement: f32 with the
  reference block test's tolerance (cosine > 0.99999, relErr < 1e-4), bf16 with the bf16 block test's
  (update cosine >= 0.9999, max-abs-rel < 1e-2).
- whole steps against oracle.step_reference: f32 on a tiny model (cosine > 0.99999, relErr < 1e-4); bf16 on a
  small model with 128-wide heads (velocity cosine >= 0.9999, max-abs-rel < 1e-2, the north star's bound; measured
  2.0e-3 with bf16 activations at every GEMM input across 4 blocks, against float64).
- the text cache gives the same velocity bit for bit; the device Euler step equals the f32 formula.
"""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, make_block, make_step, randn

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("h,w", [(4, 6), (3, 5), (5, 7), (8, 8), (128, 128)])
@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_patchify_unpatchify_bit_exact(we, graph, h, w, dt):
    T = we.transformer
    lat = np.sin(np.arange(16 * h * w) * 0.37).astype(np.float32) * 3
    if dt == "bf16":
        lat = bf16_round(lat)
    rows, cols = T.patch_grid(h, w)
    es = 2 if dt == "bf16" else 4
    mark = graph.mark()
    src = graph.buffer(bf16(lat) if dt == "bf16" else lat)
    tok = graph.buffer(rows * cols * 64 * es)
    back = graph.buffer(16 * h * w * 4)
    T.patchify(graph, src, h, w, tok, 16, dt, dt)
    T.unpatchify(graph, tok, h, w, back, 16, dt, "f32")
    raw = graph.read(tok, rows * cols * 64 * es)
    got = O.bf16_to_f32(raw.view(np.uint16)) if dt == "bf16" else raw.view(np.float32)
    again = graph.read(back, 16 * h * w * 4, np.float32).copy()
    graph.release(mark)
    assert np.array_equal(got, O.patchify(lat, h, w))
    assert np.array_equal(again, lat)


def test_patchify_rejects_bad_shapes(we, graph):
    b = graph.buffer(64)
    with pytest.raises(we._lib.WeError, match="positive"):
        we.transformer.patchify(graph, b, 0, 4, b)


def _double_case(we, graph, cfg, text, side, seed, dtype, per_channel=False):
    tokens = text + side * side
    axes = (8, 12, 12) if cfg.head_dim == 32 else (16, 56, 56)
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(text, side, side), axes, 1e4)
    ht, dt_ = make_block(we, graph, cfg, seed, per_channel)
    hi, di = make_block(we, graph, cfg, seed + 77, per_channel)
    x, temb = randn(tokens * cfg.hidden, seed + 1, 1.0), randn(6 * cfg.hidden, seed + 2, 0.3)
    want = O.joint_block_reference(x.reshape(tokens, -1), [(0, text, ht), (text, tokens - text, hi)], vars(cfg), temb,
                                   cos, sin)
    mark = graph.mark()
    rope = we.Rope(graph.buffer(cos), graph.buffer(sin), pairs, tokens)
    out = we.blocks.double_block(graph, dt_, di, cfg, graph.buffer(x), text, graph.buffer(temb), rope, dtype=dtype)
    got = graph.read(out, tokens * cfg.hidden * 4, np.float32).reshape(tokens, -1).copy()
    assert graph.device_error() == 0
    graph.release(mark)
    return x.reshape(tokens, -1), got, want


def test_double_block_f32(we, graph):
    cfg = we.blocks.BlockConfig(hidden=64, mlp=96, heads=2, kv_heads=1, head_dim=32, mlp_act="gelu", attn_gate=False)
    _, got, want = _double_case(we, graph, cfg, 5, 4, 300, "f32")
    c = O.compare(got.ravel(), want.ravel())
    assert c["cosine"] > 0.99999 and c["relativeError"] < 1e-4, c


@pytest.mark.parametrize("mlp_act,gate", [("gelu", False), ("swiglu", True)])
def test_double_block_bf16(we, graph, mlp_act, gate):
    cfg = we.blocks.BlockConfig(hidden=512, mlp=2048, heads=4, kv_heads=4, head_dim=128, mlp_act=mlp_act,
                                attn_gate=gate)
    x, got, want = _double_case(we, graph, cfg, 24, 18, 400, "bf16", per_channel=True)
    delta, wdelta = got - x, want - x
    c = O.compare(delta.ravel(), wdelta.ravel())
    rel = float(np.max(np.abs(delta - wdelta)) / np.max(np.abs(wdelta)))
    assert c["cosine"] >= 0.9999 and rel < 1e-2, (c, rel)


@pytest.mark.parametrize("text,side,images,pair", [(64, 16, 1, "0"), (256, 16, 2, "2"), (64, 8, 3, "0")],
                         ids=["1sm", "pair-2img", "3img"])
@pytest.mark.parametrize("mlp_act,gate", [("gelu", False), ("swiglu", True)])
def test_double_block_two_weight_sets_equal_per_part(we, graph, monkeypatch, text, side, images, pair, mlp_act, gate):
    """A double block's text and image rows (for every image of a batch) run each linear as ONE GEMM whose token
    tiles pick the text or image weights, scales and gates (we_gemm_fp8 row segments); the result equals the
    per-part GEMMs bit for bit, with fused q/k/v and GQA."""
    monkeypatch.setenv("WE_TC_2SM", pair)
    cfg = we.blocks.BlockConfig(hidden=512, mlp=2048, heads=4, kv_heads=2, head_dim=128, mlp_act=mlp_act,
                                attn_gate=gate)
    T = text + side * side
    R = images * T
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(text, side, side), (16, 56, 56), 1e4)
    _, dt_ = make_block(we, graph, cfg, 600, True)
    _, di = make_block(we, graph, cfg, 677, False)
    x, temb = randn(R * cfg.hidden, 601, 1.0), randn(6 * cfg.hidden, 602, 0.3)
    parts = [p for i in range(images) for p in (we.blocks.Part(i * T, text, dt_), we.blocks.Part(i * T + text,
                                                                                              T - text, di))]
    assert we.blocks._weight_plan(parts, R)[0] == "two"
    xb, tb = graph.buffer(x), graph.buffer(temb)
    rope = we.Rope(graph.buffer(np.tile(cos, images)), graph.buffer(np.tile(sin, images)), pairs, R)

    def run():
        mark = graph.mark()
        out = we.blocks.joint_block(graph, parts, cfg, xb, tb, rope, "bf16", images=images)
        got = graph.read(out, R * cfg.hidden * 4, np.float32).copy()
        graph.release(mark)
        return got

    grouped = run()
    monkeypatch.setattr(we.blocks, "_weight_plan", lambda parts, t: None)
    per_part = run()
    assert np.array_equal(grouped, per_part)
    assert graph.device_error() == 0


@pytest.mark.parametrize("images", [1, 2])
def test_deferred_residual_chain_is_bit_identical(we, graph, images):
    """Chained bf16 blocks (a double block, then a single block) with the first block's output left as a Residual
    (x1, dn) that the second block's first norm pass adds (we_add_norm_split): the second block's output, and its
    input rows, equal the plain chain (add, then norm + split) bit for bit."""
    cfg = we.blocks.BlockConfig(hidden=512, mlp=2048, heads=4, kv_heads=4, head_dim=128, mlp_act="gelu",
                                attn_gate=False)
    text, side = 24, 8
    T = text + side * side
    R = images * T
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(text, side, side), (16, 56, 56), 1e4)
    _, dt_ = make_block(we, graph, cfg, 700, True)
    _, di = make_block(we, graph, cfg, 701, True)
    _, ds = make_block(we, graph, cfg, 702, True)
    x, temb = randn(R * cfg.hidden, 703, 1.0), randn(6 * cfg.hidden, 704, 0.3)
    xb, tb = graph.buffer(x), graph.buffer(temb)
    rope = we.Rope(graph.buffer(np.tile(cos, images)), graph.buffer(np.tile(sin, images)), pairs, R)
    double = [p for i in range(images) for p in (we.blocks.Part(i * T, text, dt_), we.blocks.Part(i * T + text,
                                                                                              T - text, di))]
    single = [we.blocks.Part(0, R, ds)]

    def chain(defer):
        mark = graph.mark()
        mid = we.blocks.joint_block(graph, double, cfg, xb, tb, rope, "bf16", images=images, defer=defer)
        assert isinstance(mid, we.blocks.Residual) == defer
        out = we.blocks.joint_block(graph, single, cfg, mid, tb, rope, "bf16", images=images)
        got = graph.read(out, R * cfg.hidden * 4, np.float32).copy()
        graph.release(mark)
        return got

    plain, deferred = chain(False), chain(True)
    assert np.isfinite(plain).all() and np.array_equal(plain, deferred)
    assert graph.device_error() == 0


def test_deferred_residual_into_an_f32_block(we, graph):
    """A bf16 block's deferred Residual handed to the f32 path: the f32 block adds x1 + dn first, so its output
    equals the one it gives on the bf16 block's plain output, bit for bit."""
    cfg = we.blocks.BlockConfig(hidden=256, mlp=1024, heads=2, kv_heads=2, head_dim=128, mlp_act="gelu",
                                attn_gate=False)
    tokens = 40
    cos, sin, pairs = we.kernels.rope_tables(we.kernels.positions(8, 4, 8), (16, 56, 56), 1e4)
    _, d1 = make_block(we, graph, cfg, 720, True)
    _, d2 = make_block(we, graph, cfg, 721, True)
    x, temb = randn(tokens * cfg.hidden, 722, 1.0), randn(6 * cfg.hidden, 723, 0.3)
    xb, tb = graph.buffer(x), graph.buffer(temb)
    rope = we.Rope(graph.buffer(cos), graph.buffer(sin), pairs, tokens)
    outs = []
    for defer in (False, True):
        mark = graph.mark()
        mid = we.blocks.joint_block(graph, [we.blocks.Part(0, tokens, d1)], cfg, xb, tb, rope, "bf16", defer=defer)
        out = we.blocks.joint_block(graph, [we.blocks.Part(0, tokens, d2)], cfg, mid, tb, rope, "f32")
        outs.append(graph.read(out, tokens * cfg.hidden * 4, np.float32).copy())
        graph.release(mark)
    assert np.isfinite(outs[0]).all() and np.array_equal(outs[0], outs[1])
    assert graph.device_error() == 0


def _step_case(we, graph, scfg, h, w, text, seed, dtype, per_channel=False):
    T = we.transformer
    host, wts = make_step(we, graph, scfg, seed, per_channel)
    lat = randn(scfg.channels * h * w, seed + 5)
    ctx = randn(text * scfg.ctx_dim, seed + 6)
    if dtype == "bf16":
        lat, ctx = bf16_round(lat), bf16_round(ctx)
    want = O.step_reference(lat, h, w, 0.63, ctx, host, {**vars(scfg.block), "axes": scfg.axes, "theta": scfg.theta,
                                                          "channels": scfg.channels, "time_dim": scfg.time_dim})
    conv = bf16 if dtype == "bf16" else (lambda a: a)
    mark = graph.mark()
    inp = T.StepInputs(graph.buffer(conv(lat)), h, w, 0.63, graph.buffer(conv(ctx)), text)
    vel, txt = T.transformer(graph, wts, scfg, inp, dtype=dtype)
    got = graph.read(vel, scfg.channels * h * w * 4, np.float32).copy()
    inp.text_cache = txt
    vel2, _ = T.transformer(graph, wts, scfg, inp, dtype=dtype)
    again = graph.read(vel2, scfg.channels * h * w * 4, np.float32).copy()
    assert graph.device_error() == 0
    graph.release(mark)
    return got, again, want


def test_step_f32_matches_the_float64_step(we, graph):
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=64, mlp=128, heads=2, kv_heads=2, head_dim=32, mlp_act="gelu", attn_gate=False)
    scfg = T.StepConfig(block=bc, double=1, single=2, ctx_dim=48, axes=(8, 12, 12))
    got, again, want = _step_case(we, graph, scfg, 6, 10, 5, 500, "f32")
    c = O.compare(got, want)
    assert c["cosine"] > 0.99999 and c["relativeError"] < 1e-4, c
    assert np.array_equal(got, again)


def test_step_bf16_matches_the_float64_step(we, graph):
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=256, mlp=1024, heads=2, kv_heads=2, head_dim=128, mlp_act="gelu",
                               attn_gate=False)
    scfg = T.StepConfig(block=bc, double=2, single=2, ctx_dim=256)
    got, again, want = _step_case(we, graph, scfg, 16, 18, 8, 600, "bf16", per_channel=True)
    c = O.compare(got, want)
    rel = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    print(f"small bf16 step vs float64: cosine {c['cosine']:.7f}, max-abs-rel {rel:.2e}")
    assert c["cosine"] >= 0.9999 and rel < 1e-2, (c, rel)
    assert np.array_equal(got, again)


def test_euler_step_on_device(we, graph):
    T = we.transformer
    x, v = randn(1000, 1), randn(1000, 2)
    s = T.sigmas(4)
    mark = graph.mark()
    out = T.euler_step(graph, graph.buffer(x), graph.buffer(v), s[1], s[2], 1000)
    got = graph.read(out, 4000, np.float32).copy()
    graph.release(mark)
    want = O.euler_step(x, v, s[1], s[2])
    assert np.max(np.abs(got - want)) <= 2 * np.spacing(np.abs(want).max())


def test_batch_of_images_equals_one_at_a_time(we, graph):
    """A batch runs as one token stream (one GEMM per linear over all images' rows, attention per image): each
    image's velocity matches the single-image step and the float64 step."""
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=256, mlp=1024, heads=2, kv_heads=2, head_dim=128, mlp_act="gelu",
                               attn_gate=False)
    scfg = T.StepConfig(block=bc, double=1, single=2, ctx_dim=256)
    h, w, text = 12, 14, 8
    host, wts = make_step(we, graph, scfg, 700, per_channel=True)
    cfgd = {**vars(bc), "axes": scfg.axes, "theta": scfg.theta, "channels": scfg.channels, "time_dim": scfg.time_dim}
    lats = [bf16_round(randn(16 * h * w, 710 + i)) for i in range(3)]
    ctxs = [bf16_round(randn(text * 256, 720 + i)) for i in range(3)]
    mark = graph.mark()
    inputs = [T.StepInputs(graph.buffer(bf16(l)), h, w, 0.41, graph.buffer(bf16(c)), text) for l, c in zip(lats, ctxs)]
    vel, txts = T.transformer(graph, wts, scfg, inputs, dtype="bf16")
    got = [graph.read(v, 16 * h * w * 4, np.float32).copy() for v in vel]
    single = []
    for ib in inputs:
        v1, _ = T.transformer(graph, wts, scfg, ib, dtype="bf16")
        single.append(graph.read(v1, 16 * h * w * 4, np.float32).copy())
    assert graph.device_error() == 0
    graph.release(mark)
    for i in range(3):
        assert np.allclose(got[i], single[i], rtol=1e-5, atol=1e-6 * np.abs(single[i]).max())
        want = O.step_reference(lats[i], h, w, 0.41, ctxs[i], host, cfgd)
        c = O.compare(got[i], want)
        assert c["cosine"] >= 0.9999, c


def test_sampling_loop_matches_the_float64_loop(we, graph):
    """Two Euler steps (src/pipeline/generate.ts:94-105) of a tiny f32 model against the float64 step + eulerStep."""
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=64, mlp=128, heads=2, kv_heads=2, head_dim=32, mlp_act="gelu", attn_gate=False)
    scfg = T.StepConfig(block=bc, double=1, single=1, ctx_dim=32, axes=(8, 12, 12))
    h, w, text = 6, 8, 4
    host, wts = make_step(we, graph, scfg, 800)
    cfgd = {**vars(bc), "axes": scfg.axes, "theta": scfg.theta, "channels": scfg.channels, "time_dim": scfg.time_dim}
    noise = [O.gaussian(16 * h * w, 5 + i) for i in range(2)]
    ctxs = [randn(text * 32, 810 + i) for i in range(2)]
    mark = graph.mark()
    out = T.sample(graph, wts, scfg, [graph.buffer(z) for z in noise], [graph.buffer(c) for c in ctxs], h, w, text,
                   steps=2, dtype="f32")
    got = [graph.read(o, 16 * h * w * 4, np.float32).copy() for o in out]
    graph.release(mark)
    sig = O.sigmas(2)
    for i in range(2):
        x = noise[i]
        for s in range(2):
            v = O.step_reference(x, h, w, sig[s], ctxs[i], host, cfgd)
            x = O.euler_step(x, v, sig[s], sig[s + 1])
        c = O.compare(got[i], x)
        assert c["cosine"] > 0.99999 and c["relativeError"] < 1e-4, c


@pytest.mark.parametrize("slots", [2, 3])
def test_streamed_weights_step_equals_the_resident_step(we, graph, slots):
    """Block weights streamed from pinned host memory one layer ahead (StreamedBlocks over we_streamer: 2 or 3 device
    slots, layers larger than a slot's share refilled while earlier blocks run) give the resident step's velocity
    bit for bit, for a batch of 2 images and for a 2-step sampling loop; every step copies every layer."""
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=512, mlp=2048, heads=4, kv_heads=4, head_dim=128, mlp_act="gelu",
                               attn_gate=False)
    scfg = T.StepConfig(block=bc, double=2, single=3, ctx_dim=256)
    h, w, text = 16, 16, 8
    _, wts = make_step(we, graph, scfg, 900, per_channel=True)
    lats = [bf16_round(randn(16 * h * w, 910 + i)) for i in range(2)]
    ctxs = [bf16_round(randn(text * 256, 920 + i)) for i in range(2)]
    mark = graph.mark()
    inputs = [T.StepInputs(graph.buffer(bf16(l)), h, w, 0.55, graph.buffer(bf16(c)), text) for l, c in zip(lats, ctxs)]
    vel, _ = T.transformer(graph, wts, scfg, inputs, dtype="bf16")
    want = [graph.read(v, 16 * h * w * 4, np.float32).copy() for v in vel]
    st = T.StreamedBlocks(graph, wts, slots=slots)
    try:
        for _ in range(2):  # a second pass wraps around the layers again
            vel, _ = T.transformer(graph, wts, scfg, inputs, dtype="bf16", streamed=st)
            got = [graph.read(v, 16 * h * w * 4, np.float32).copy() for v in vel]
            assert all(np.array_equal(a, b) for a, b in zip(got, want))
        noise = [graph.buffer(randn(16 * h * w, 930 + i)) for i in range(2)]
        ctxb = [graph.buffer(bf16(c)) for c in ctxs]
        res = T.sample(graph, wts, scfg, noise, ctxb, h, w, text, steps=2, dtype="bf16")
        stm = T.sample(graph, wts, scfg, noise, ctxb, h, w, text, steps=2, dtype="bf16", streamed=st)
        for a, b in zip(res, stm):
            assert np.array_equal(graph.read(a, 16 * h * w * 4, np.float32), graph.read(b, 16 * h * w * 4, np.float32))
        layers = scfg.double + scfg.single
        # 4 passes over 5 layers: every layer is copied in every pass except those still in a slot from the pass before
        assert st.stats["copies"] >= 4 * layers - slots
    finally:
        st.close()
    assert graph.device_error() == 0
    graph.release(mark)
