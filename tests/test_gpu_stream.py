"""Layer streaming (we_streamer_*): weights copied from host memory into a ring of device slots on a
side stream while the context stream computes; results must equal the resident-weight results."""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, fast_fp8, randn

pytestmark = pytest.mark.gpu


def test_streamed_layers_match_resident_weights(we):
    g = we.Graph(0)
    try:
        layers, n, k, m, slots = 6, 384, 512, 64, 2
        ws = [fast_fp8(n * k, 100 + l) for l in range(layers)]
        scales = [(np.abs(randn(n, 200 + l, 0.01)) + np.float32(1e-3)).astype(np.float32) for l in range(layers)]
        x = bf16_round(randn(m * k, 7))
        xb = g.buffer(bf16(x))
        sb = [g.buffer(s) for s in scales]
        want = [O.matmul(x, O.FP8, ws[l], m, n, k, chan_scale=scales[l]) for l in range(layers)]
        with we.Streamer(g, ws, slots=slots) as st:
            for step in range(2):
                outs = []
                for l in range(layers):
                    w = st.acquire(l)
                    y = g.buffer(m * n * 4)
                    we.kernels.matmul(g, xb, w, y, m, n, k, 1.0, x_dtype="bf16", w_dtype="fp8", chan_scale=sb[l])
                    st.release(l)
                    outs.append(y)
                for l in range(layers):
                    got = g.read(outs[l], m * n * 4, np.float32)
                    assert O.rel_error(got, want[l]) < 1e-5, (step, l)
            s = st.stats
            assert s["copies"] >= 2 * layers and s["bytesCopied"] == s["copies"] * n * k
        assert g.device_error() == 0
    finally:
        g.destroy()


def test_streamer_refuses_a_busy_slot(we):
    g = we.Graph(0)
    try:
        ws = [np.full(4096, l, np.uint8) for l in range(4)]
        with we.Streamer(g, ws, slots=2) as st:
            st.acquire(0)
            with pytest.raises(we._lib.WeError, match="release it first"):
                st.acquire(2)  # same slot as layer 0, which is still held
            st.release(0)
            d = st.acquire(2)
            assert g.read(d, 4096)[0] == 2
            st.release(2)
            with pytest.raises(we._lib.WeError, match="not acquired"):
                st.release(2)
    finally:
        g.destroy()
