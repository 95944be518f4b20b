"""Shared helpers of the GPU parity tests (inputs from the reference tests' generators)."""
import math

import numpy as np

from oracle import oracle as O


def lcg_floats(n, seed, size=1.0, centred=True):
    r = O.lcg(seed)
    if centred:
        return np.array([(r() * 2 - 1) * size for _ in range(n)], np.float32)
    return np.array([r() * size for _ in range(n)], np.float32)


def lcg_fp8(n, seed):
    """Any fp8 byte except the NaN codes (tests/gpu/matmul.test.ts:17-21)."""
    r = O.lcg(seed)
    out = np.empty(n, np.uint8)
    for i in range(n):
        b = math.floor(r() * 256)
        out[i] = b - 1 if (b & 0x7F) == 0x7F else b
    return out


def fast_fp8(n, seed):
    """Random non-NaN e4m3 bytes for large cases (numpy generator; the oracle decodes them)."""
    b = np.random.default_rng(seed).integers(0, 256, n, dtype=np.uint8)
    b[(b & 0x7F) == 0x7F] -= 1
    return b


def randn(n, seed, std=1.0):
    return (np.random.default_rng(seed).standard_normal(n) * std).astype(np.float32)


def bf16(x):
    """bf16 bits (uint16) of float32 values, RNE."""
    return O.bf16_bits(np.asarray(x, np.float32))


def bf16_round(x):
    return O.bf16_round(np.asarray(x, np.float32))


def max_err(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)))) if np.size(a) else 0.0


def make_linear(we, graph, n, k, seed, per_channel=True, std=0.02):
    """A random fp8 linear on the device and its host dict for the float64 oracle. per_channel: N(0, std)
    weights quantised with per-output-channel absmax scales; else random e4m3 bytes with a scalar scale."""
    if per_channel:
        q, s = O.quant_fp8_channel(randn(n * k, seed, std), n, k)
        return {"bytes": q, "n": n, "k": k, "chan_scale": s}, we.Linear(graph.buffer(q), "fp8", 1.0, n, k,
                                                                         chan_scale=graph.buffer(s))
    q = fast_fp8(n * k, seed)
    sc = 0.002 if k <= 512 else 0.002 * (512 / k) ** 0.5
    return {"bytes": q, "n": n, "k": k, "scale": sc}, we.Linear(graph.buffer(q), "fp8", sc, n, k)


def make_block(we, graph, cfg, seed, per_channel=False, fuse=True):
    """Random fp8 block weights on the device plus their host copies for the float64 reference."""
    hid, mlp, heads, kvh, hd = cfg.hidden, cfg.mlp, cfg.heads, cfg.kv_heads, cfg.head_dim
    shapes = {"wq": (heads * hd, hid), "wk": (kvh * hd, hid), "wv": (kvh * hd, hid), "wo": (hid, hid),
              "mlp_up": (mlp, hid), "mlp_down": (hid, mlp)}
    if cfg.attn_gate:
        shapes["gate"] = (hid, hid)
    if cfg.mlp_act == "swiglu":
        shapes["mlp_gate"] = (mlp, hid)
    host, dev = {}, {}
    for i, (name, (n, k)) in enumerate(sorted(shapes.items())):
        host[name], dev[name] = make_linear(we, graph, n, k, seed + i, per_channel)
    vec = {"norm1": randn(hid, seed + 50, 0.5), "norm2": randn(hid, seed + 51, 0.5), "norm_q": randn(hd, seed + 52, 0.5),
           "norm_k": randn(hd, seed + 53, 0.5), "table": randn(6 * hid, seed + 54, 0.3)}
    host.update(vec)
    bw = we.blocks.BlockWeights(**dev, **{k: graph.buffer(v) for k, v in vec.items()})
    return host, (we.blocks.fuse_qkv(graph, bw) if fuse else bw)


def make_step(we, graph, scfg, seed, per_channel=False):
    """Random weights of a whole step model (Flux-style layout) on the device plus host copies for
    oracle.step_reference. The edge linears (time MLP, text, first, last) are per-channel N(0, 0.02)."""
    bc, T = scfg.block, we.transformer
    hid, ch = bc.hidden, scfg.channels
    host, dev = {}, {}
    for i, (name, (n, k)) in enumerate([("first", (hid, 4 * ch)), ("tmlp0", (hid, scfg.time_dim)),
                                        ("tmlp2", (hid, hid)), ("tproj", (6 * hid, hid)),
                                        ("txt_in", (hid, scfg.ctx_dim)), ("last_linear", (4 * ch, hid))]):
        host[name], dev[name] = make_linear(we, graph, n, k, seed + i, True)
    host["double"], dev["double"] = [], []
    for i in range(scfg.double):
        ht, dt = make_block(we, graph, bc, seed + 1000 + 200 * i, per_channel)
        hi, di = make_block(we, graph, bc, seed + 1100 + 200 * i, per_channel)
        host["double"].append((ht, hi))
        dev["double"].append((dt, di))
    host["single"], dev["single"] = [], []
    for i in range(scfg.single):
        hb, db = make_block(we, graph, bc, seed + 9000 + 100 * i, per_channel)
        host["single"].append(hb)
        dev["single"].append(db)
    for i, name in enumerate(("last_norm", "last_scale", "last_shift")):
        host[name] = randn(hid, seed + 60 + i, 0.3)
        dev[name] = graph.buffer(host[name])
    return host, T.TransformerWeights(**dev)

