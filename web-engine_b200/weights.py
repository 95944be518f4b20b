"""Model weights from .safetensors files: the loader of src/weights/ and src/model/weights.ts over the native reader.

    read_header(path)                      readHeader (src/weights/safetensors.ts:27-64), native: we_st_open
    Safetensors.read(name, limit)          readTensor (safetensors.ts:67-70)
    Safetensors.upload(graph, name)        file -> pinned staging -> HBM (we_st_upload)
    to_float32(dtype, data)                toFloat32 (src/weights/fp8.ts:37-53)
    fp8_weights(st), block_groups(names)   src/weights/inspect.ts:9-31
    load_linear(graph, st, name)           loadLinear (src/model/weights.ts:26-50)
    load_floats(st, name)                  loadFloats (weights.ts:53-56)
    load_block(graph, st, prefix)          loadAttentionMlp + the block's modulation table (weights.ts:70-91)
    write_safetensors(path, tensors)       the file layout the Python library writes (exports, test fixtures)

Names follow the reference's ComfyUI Krea 2 files ("blocks.N.attn.wq", "blocks.N.prenorm.scale", ...).
"""
from __future__ import annotations

import ctypes as C
import json
import re
import struct
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .graph import Buffer, Graph
from .ops import Linear

DTYPE_BYTES = {"F64": 8, "F32": 4, "F16": 2, "BF16": 2, "F8_E4M3": 1, "F8_E5M2": 1, "I64": 8, "I32": 4, "I16": 2,
               "I8": 1, "U64": 8, "U32": 4, "U16": 2, "U8": 1, "BOOL": 1}


class SafetensorsError(ValueError):
    """A broken or hostile file (SafetensorsError, safetensors.ts:18-20)."""


@dataclass(frozen=True)
class TensorInfo:
    name: str
    dtype: str
    shape: tuple
    offset: int  # absolute byte offset in the file
    size: int    # bytes


def _info(t: L.StTensor) -> TensorInfo:
    return TensorInfo(t.name.decode(), t.dtype.decode(), tuple(t.shape[i] for i in range(min(t.ndim, 8))), t.offset,
                      t.size)


class Safetensors:
    """An open .safetensors file: `tensors` (name -> TensorInfo, header order) and `metadata`."""

    def __init__(self, path: str):
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        rc = L.lib().we_st_open(str(path).encode(), C.byref(h), err, len(err))
        if rc == L.WE_EIO:
            raise OSError(err.value.decode())
        if rc != L.WE_OK:
            raise SafetensorsError(err.value.decode())
        self._h = h
        t = L.StTensor()
        self.tensors = {}
        for i in range(L.lib().we_st_count(h)):
            L.lib().we_st_tensor_at(h, i, C.byref(t))
            info = _info(t)
            self.tensors[info.name] = info
        self.metadata = {}
        k, v = C.c_char_p(), C.c_char_p()
        for i in range(L.lib().we_st_metadata_count(h)):
            L.lib().we_st_metadata_at(h, i, C.byref(k), C.byref(v))
            self.metadata[k.value.decode()] = v.value.decode()

    def tensor(self, name: str) -> TensorInfo:
        t = self.tensors.get(name)
        if t is None:
            raise KeyError(f"Missing tensor {name}: is this a Krea 2 file?")
        return t

    def read(self, name: str, limit: int | None = None) -> np.ndarray:
        """The raw bytes of one tensor (or only its first `limit` bytes)."""
        t = self.tensor(name)
        n = t.size if limit is None else min(limit, t.size)
        out = np.empty(n, np.uint8)
        rc = L.lib().we_st_read(self._h, name.encode(), out.ctypes.data_as(C.c_void_p), n)
        if rc != L.WE_OK:
            raise SafetensorsError(f"cannot read {name}")
        return out

    def upload(self, graph: Graph, name: str, dst=None) -> Buffer:
        """The tensor's bytes in a device buffer (a new one from the graph unless `dst` is given)."""
        t = self.tensor(name)
        out = dst if dst is not None else graph.buffer(t.size)
        L.check(graph.ctx, L.lib().we_st_upload(graph.ctx, self._h, name.encode(),
                                                C.c_void_p(out.ptr if hasattr(out, "ptr") else out.data_ptr())))
        return out

    def close(self) -> None:
        if self._h:
            L.lib().we_st_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 (interpreter shutdown)
            pass


def read_header(path: str) -> Safetensors:
    return Safetensors(path)


# ---------------- decoding (src/weights/fp8.ts) ----------------
def _fp8_table(exp_bits: int, bias: int, ieee_special: bool) -> np.ndarray:
    """All 256 codes of an 8-bit float: sign, exp_bits exponent bits, the rest mantissa (fp8.ts:4-23)."""
    man_bits = 7 - exp_bits
    b = np.arange(256)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> man_bits) & ((1 << exp_bits) - 1)
    m = b & ((1 << man_bits) - 1)
    scale = float(1 << man_bits)
    val = np.where(e == 0, sign * (m / scale) * 2.0 ** (1 - bias), sign * (1 + m / scale) * 2.0 ** (e - bias))
    top = (1 << exp_bits) - 1
    if ieee_special:  # e5m2: all-ones exponent is inf / NaN
        val = np.where(e == top, np.where(m == 0, sign * np.inf, np.nan), val)
    else:  # e4m3fn: only S.1111.111 is NaN
        val = np.where((e == top) & (m == (1 << man_bits) - 1), np.nan, val)
    return val.astype(np.float32)


E4M3 = _fp8_table(4, 7, False)
E5M2 = _fp8_table(5, 15, True)


def to_float32(dtype: str, data) -> np.ndarray:
    """Little-endian tensor bytes -> float32 (toFloat32, fp8.ts:37-53)."""
    raw = np.frombuffer(bytes(data), np.uint8)
    if dtype == "F32":
        return raw.view(np.float32).copy()
    if dtype == "BF16":
        return (raw.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
    if dtype == "F16":
        return raw.view(np.float16).astype(np.float32)
    if dtype == "F8_E4M3":
        return E4M3[raw]
    if dtype == "F8_E5M2":
        return E5M2[raw]
    raise ValueError(f"Can't decode {dtype} as floats")


# ---------------- inspection (src/weights/inspect.ts) ----------------
SCALE_SUFFIXES = (".scale_weight", ".weight_scale")


def fp8_weights(st: Safetensors) -> list:
    """fp8 ".weight" tensors with their per-layer scale tensor or None (ComfyUI fp8_scaled; inspect.ts:9-19),
    sorted by name."""
    out = []
    for t in st.tensors.values():
        if not t.dtype.startswith("F8_") or not t.name.endswith(".weight"):
            continue
        base = t.name[: -len(".weight")]
        scale = next((st.tensors[base + s] for s in SCALE_SUFFIXES if base + s in st.tensors), None)
        out.append((t, scale))
    return sorted(out, key=lambda p: p[0].name)


def block_groups(names) -> list:
    """Repeated blocks ("x.blocks.0.…") and how many of each, biggest first (inspect.ts:22-31)."""
    groups: dict = {}
    for name in names:
        m = re.match(r"^(.*?)\.(\d+)\.", name)
        if m:
            groups.setdefault(m.group(1), set()).add(m.group(2))
    return sorted(((p, len(ids)) for p, ids in groups.items()), key=lambda g: -g[1])


# ---------------- loading (src/model/weights.ts) ----------------
def load_floats(st: Safetensors, name: str) -> np.ndarray:
    """Any float tensor as f32 on the host (norm weights, modulation tables; weights.ts:53-56)."""
    t = st.tensor(name)
    return to_float32(t.dtype, st.read(name))


def load_linear(graph: Graph, st: Safetensors, name: str) -> Linear:
    """A linear layer as stored (loadLinear, weights.ts:26-50): fp8 [n, k] with its weight_scale (or ComfyUI's
    scale_weight) or bf16 [n, k], plus its bias if present. The weight bytes go straight to HBM (we_st_upload).
    A scale tensor of n values is used per output channel, one value as the scalar scale."""
    w = st.tensor(f"{name}.weight")
    if len(w.shape) != 2 or w.dtype not in ("F8_E4M3", "BF16"):
        raise SafetensorsError(f"{name}.weight: expected a 2D F8_E4M3 or BF16 tensor, got {w.dtype} {list(w.shape)}")
    n, k = w.shape
    buf = st.upload(graph, w.name)
    bias = graph.buffer(load_floats(st, f"{name}.bias")) if f"{name}.bias" in st.tensors else None
    if w.dtype == "BF16":
        return Linear(buf, "bf16", 1.0, n, k, bias=bias)
    sname = next((name + s for s in (".weight_scale", ".scale_weight") if name + s in st.tensors), None)
    if sname is None:
        raise KeyError(f"Missing tensor {name}.weight_scale: is this a Krea 2 file?")
    scale = load_floats(st, sname)
    if scale.size == n and n > 1:
        return Linear(buf, "fp8", 1.0, n, k, bias=bias, chan_scale=graph.buffer(scale.astype(np.float32)))
    return Linear(buf, "fp8", float(scale[0]), n, k, bias=bias)


def load_block(graph: Graph, st: Safetensors, prefix: str, gate: bool = True, mlp_gate: bool = True):
    """One block's weights by the reference's names (loadAttentionMlp + loadBlock, weights.ts:70-91): attn.wq/wk/wv/
    gate/wo, mlp.gate/up/down, prenorm/postnorm scales, qk-norm scales and the modulation table mod.lin."""
    from .block import BlockWeights, fuse_qkv

    lin = lambda n: load_linear(graph, st, f"{prefix}.{n}")  # noqa: E731
    vec = lambda n: graph.buffer(load_floats(st, f"{prefix}.{n}"))  # noqa: E731
    return fuse_qkv(graph, BlockWeights(wq=lin("attn.wq"), wk=lin("attn.wk"), wv=lin("attn.wv"), wo=lin("attn.wo"),
                        mlp_up=lin("mlp.up"), mlp_down=lin("mlp.down"), norm1=vec("prenorm.scale"),
                        norm2=vec("postnorm.scale"), norm_q=vec("attn.qknorm.qnorm.scale"),
                        norm_k=vec("attn.qknorm.knorm.scale"), table=vec("mod.lin"),
                        gate=lin("attn.gate") if gate else None, mlp_gate=lin("mlp.gate") if mlp_gate else None))


# ---------------- writing ----------------
def write_safetensors(path: str, tensors: dict, metadata: dict | None = None) -> None:
    """Writes {name: (dtype, shape, bytes)} in header order, data packed back to back (the layout the Python
    library writes: 8-byte little-endian header size, JSON header, data)."""
    header: dict = {"__metadata__": dict(metadata)} if metadata else {}
    off = 0
    blobs = []
    for name, (dtype, shape, data) in tensors.items():
        b = bytes(data)
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(b)]}
        off += len(b)
        blobs.append(b)
    text = json.dumps(header, separators=(",", ":")).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(text)))
        f.write(text)
        for b in blobs:
            f.write(b)


def load_model(graph: Graph, st: Safetensors, cfg) -> "object":
    """The step model's weights (loadTransformer, weights.ts:94-131, for the Flux-style layout of the step driver):
    first, tmlp.0, tmlp.2, tproj.1, txt_in, last.linear; last.norm.scale and last.modulation.lin [2, hidden]
    (scale, shift); double blocks under "double_blocks.N.txt" / "double_blocks.N.img", single blocks under
    "blocks.N" (the reference's names inside each block)."""
    from .transformer import TransformerWeights

    bc = cfg.block
    opts = {"gate": bc.attn_gate, "mlp_gate": bc.mlp_act == "swiglu"}
    last = load_floats(st, "last.modulation.lin")
    hidden = last.size // 2
    if hidden != bc.hidden:
        raise SafetensorsError(f"last.modulation.lin: hidden {hidden} does not match the config's {bc.hidden}")
    return TransformerWeights(
        first=load_linear(graph, st, "first"), tmlp0=load_linear(graph, st, "tmlp.0"),
        tmlp2=load_linear(graph, st, "tmlp.2"), tproj=load_linear(graph, st, "tproj.1"),
        txt_in=load_linear(graph, st, "txt_in"),
        double=[(load_block(graph, st, f"double_blocks.{i}.txt", **opts),
                 load_block(graph, st, f"double_blocks.{i}.img", **opts)) for i in range(cfg.double)],
        single=[load_block(graph, st, f"blocks.{i}", **opts) for i in range(cfg.single)],
        last_norm=graph.buffer(load_floats(st, "last.norm.scale")), last_scale=graph.buffer(last[:hidden].copy()),
        last_shift=graph.buffer(last[hidden:].copy()), last_linear=load_linear(graph, st, "last.linear"))
