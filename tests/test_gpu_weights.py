"""The weight loader on the GPU: file -> pinned staging -> HBM (we_st_upload) and whole-model loading.

- a 72 MB tensor (three 32 MB staging chunks, the last partial) reaches HBM byte for byte;
- a small step model written to .safetensors (fp8 linears with weight_scale / per-channel scales, f32 vectors,
  the reference's names) loads with load_model and gives the same velocity, bit for bit, as the same weights
  uploaded directly, and matches the float64 step.
"""
import numpy as np
import pytest

from oracle import oracle as O
from util import bf16, bf16_round, make_step, randn

pytestmark = pytest.mark.gpu


def test_upload_large_tensor_in_chunks(we, graph, tmp_path):
    data = np.random.default_rng(3).integers(0, 256, 72 * 1024 * 1024 + 77, dtype=np.uint8)
    p = str(tmp_path / "big.safetensors")
    we.weights.write_safetensors(p, {"small": ("U8", [3], bytes([1, 2, 3])), "big": ("U8", [data.size], data.tobytes())})
    with we.weights.read_header(p) as st:
        mark = graph.mark()
        buf = st.upload(graph, "big")
        small = st.upload(graph, "small")
        got = graph.read(buf, data.size)
        assert np.array_equal(got, data)
        assert graph.read(small, 3).tolist() == [1, 2, 3]
        graph.release(mark)


def _linear_tensors(name, lin):
    out = {f"{name}.weight": ("F8_E4M3", [lin["n"], lin["k"]], lin["bytes"].tobytes())}
    if lin.get("chan_scale") is not None:
        out[f"{name}.weight_scale"] = ("F32", [lin["n"]], lin["chan_scale"].astype(np.float32).tobytes())
    else:
        out[f"{name}.scale_weight"] = ("F32", [], np.float32(lin["scale"]).tobytes())  # ComfyUI's other suffix
    return out


def _block_tensors(prefix, h):
    t = {}
    for key, name in (("wq", "attn.wq"), ("wk", "attn.wk"), ("wv", "attn.wv"), ("wo", "attn.wo"), ("gate", "attn.gate"),
                      ("mlp_gate", "mlp.gate"), ("mlp_up", "mlp.up"), ("mlp_down", "mlp.down")):
        if key in h:
            t.update(_linear_tensors(f"{prefix}.{name}", h[key]))
    for key, name in (("norm1", "prenorm.scale"), ("norm2", "postnorm.scale"), ("norm_q", "attn.qknorm.qnorm.scale"),
                      ("norm_k", "attn.qknorm.knorm.scale"), ("table", "mod.lin")):
        t[f"{prefix}.{name}"] = ("F32", [h[key].size], h[key].astype(np.float32).tobytes())
    return t


def _model_tensors(host):
    t = {}
    for key, name in (("first", "first"), ("tmlp0", "tmlp.0"), ("tmlp2", "tmlp.2"), ("tproj", "tproj.1"),
                      ("txt_in", "txt_in"), ("last_linear", "last.linear")):
        t.update(_linear_tensors(name, host[key]))
    for i, (ht, hi) in enumerate(host["double"]):
        t.update(_block_tensors(f"double_blocks.{i}.txt", ht))
        t.update(_block_tensors(f"double_blocks.{i}.img", hi))
    for i, hb in enumerate(host["single"]):
        t.update(_block_tensors(f"blocks.{i}", hb))
    t["last.norm.scale"] = ("F32", [host["last_norm"].size], host["last_norm"].tobytes())
    both = np.concatenate([host["last_scale"], host["last_shift"]]).astype(np.float32)
    t["last.modulation.lin"] = ("F32", [2, both.size // 2], both.tobytes())
    return t


@pytest.mark.parametrize("per_channel", [False, True])
def test_load_model_from_safetensors(we, graph, tmp_path, per_channel):
    T = we.transformer
    bc = we.blocks.BlockConfig(hidden=256, mlp=1024, heads=2, kv_heads=2, head_dim=128, mlp_act="swiglu",
                               attn_gate=True)
    scfg = T.StepConfig(block=bc, double=1, single=1, ctx_dim=256)
    h, w, text = 8, 10, 8
    host, direct = make_step(we, graph, scfg, 900, per_channel)
    p = str(tmp_path / "model.safetensors")
    we.weights.write_safetensors(p, _model_tensors(host), {"format": "pt"})
    lat, ctx = bf16_round(randn(16 * h * w, 901)), bf16_round(randn(text * 256, 902))
    with we.weights.read_header(p) as st:
        loaded = we.weights.load_model(graph, st, scfg)
    mark = graph.mark()
    outs = []
    for wts in (direct, loaded):
        inp = T.StepInputs(graph.buffer(bf16(lat)), h, w, 0.5, graph.buffer(bf16(ctx)), text)
        v, _ = T.transformer(graph, wts, scfg, inp, dtype="bf16")
        outs.append(graph.read(v, 16 * h * w * 4, np.float32).copy())
    assert graph.device_error() == 0
    graph.release(mark)
    assert np.array_equal(outs[0], outs[1])
    want = O.step_reference(lat, h, w, 0.5, ctx, host, {**vars(bc), "axes": scfg.axes, "theta": scfg.theta,
                                                         "channels": 16, "time_dim": 256})
    assert O.compare(outs[1], want)["cosine"] >= 0.9999


def test_load_linear_rejects_wrong_layouts(we, graph, tmp_path):  # src/model/weights.ts:28-30
    p = str(tmp_path / "bad.safetensors")
    we.weights.write_safetensors(p, {"a.weight": ("F32", [2, 2], bytes(16)), "b.weight": ("F8_E4M3", [4], bytes(4))})
    with we.weights.read_header(p) as st:
        with pytest.raises(we.weights.SafetensorsError, match="expected a 2D F8_E4M3 or BF16 tensor"):
            we.weights.load_linear(graph, st, "a")
        with pytest.raises(we.weights.SafetensorsError, match="expected a 2D"):
            we.weights.load_linear(graph, st, "b")
        with pytest.raises(KeyError, match="Missing tensor c.weight"):
            we.weights.load_linear(graph, st, "c")
