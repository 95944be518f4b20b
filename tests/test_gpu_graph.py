"""CUDA graphs of this library's ops (we_capture_begin / we_capture_end / we_graph_launch): a recorded sequence
replays with new inputs and gives the eager results bit for bit; a whole step's blocks captured as a StepGraph
give the eager step's velocity bit for bit, for two different latents and timesteps; synchronising calls are
refused while capturing; a capture's buffers stay out of the context's pool."""
import numpy as np
import pytest

from util import bf16, bf16_round, make_step, randn

pytestmark = pytest.mark.gpu


@pytest.fixture
def sgraph(we):
    """A context on its own stream (capture needs a non-default stream)."""
    import torch

    g = we.Graph(0)
    st = torch.cuda.Stream(device=torch.device("cuda", 0))
    g.set_stream(st.cuda_stream)
    yield g
    g.destroy()


def test_captured_ops_replay_with_new_inputs(we, sgraph):
    g = sgraph
    m, n, k = 300, 512, 256
    w = we.Linear(g.buffer(np.random.default_rng(1).integers(0, 120, n * k, dtype=np.uint8)), "fp8", 0.01, n, k)
    wn = g.buffer(randn(n, 2, 0.3))
    xin = g.buffer(m * k * 2)

    def ops(x):
        y = we.linear(g, x, w, m, x_dtype="bf16", y_dtype="bf16")
        return we.norm(g, y, wn, m, n, we.no_mod(g, n), x_dtype="bf16", out_dtype="f32")

    with g.capture() as cap:
        out = ops(xin)
    for seed in (3, 4):
        x = bf16(bf16_round(randn(m * k, seed)))
        g.write(xin, x)
        cap.launch()
        got = g.read(out, m * n * 4, np.float32).copy()
        want = g.read(ops(g.buffer(x)), m * n * 4, np.float32).copy()
        assert np.array_equal(got, want)
    assert g.device_error() == 0
    cap.destroy()


def test_capture_refuses_synchronising_calls(we, sgraph):
    g = sgraph
    b = g.buffer(64)
    with pytest.raises(we._lib.WeError, match="while capturing"):
        with g.capture():
            g.read(b, 64)
    # the context works again after the failed capture
    assert g.read(g.buffer(np.arange(4, dtype=np.float32)), 16, np.float32).tolist() == [0, 1, 2, 3]


def test_step_graph_equals_the_eager_step(we, sgraph):
    g = sgraph
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=256, mlp=1024, heads=2, kv_heads=2, head_dim=128, mlp_act="gelu",
                               attn_gate=False)
    scfg = T.StepConfig(block=bc, double=2, single=2, ctx_dim=256)
    h, w, text = 16, 18, 8
    _, wts = make_step(we, g, scfg, 1300, per_channel=True)
    sgr = T.StepGraph(g, wts, scfg, h, w, text, dtype="bf16")
    for seed, sigma in ((1, 0.9), (2, 0.35)):
        lat, ctx = bf16_round(randn(16 * h * w, 1310 + seed)), bf16_round(randn(text * 256, 1320 + seed))
        inp = T.StepInputs(g.buffer(bf16(lat)), h, w, sigma, g.buffer(bf16(ctx)), text)
        v1, _ = T.transformer(g, wts, scfg, inp, dtype="bf16")
        v2, _ = T.transformer(g, wts, scfg, inp, dtype="bf16", captured=sgr)
        a = g.read(v1, 16 * h * w * 4, np.float32).copy()
        b = g.read(v2, 16 * h * w * 4, np.float32).copy()
        assert np.array_equal(a, b)
    with pytest.raises(ValueError, match="another geometry"):
        T.transformer(g, wts, scfg, T.StepInputs(g.buffer(64), 8, 8, 0.5, g.buffer(64), text), dtype="bf16",
                      captured=sgr)
    assert g.device_error() == 0
    sgr.destroy()
