"""The .safetensors reader (native we_st_*) and the loader's host functions, no GPU.

Mirrors tests/safetensors.test.ts case by case (absolute offsets, one tensor's bytes, empty file, every
hostile-file rejection with its message, readTensor with a limit), plus a deeply nested header, the decoders
against the oracle (src/weights/fp8.ts), the fp8_scaled pairing and block groups (src/weights/inspect.ts).
"""
import struct

import numpy as np
import pytest

from oracle import oracle as O


def raw(tmp_path, header_text: str, data: bytes = b"", size_override=None, name="f.safetensors"):
    """An 8-byte size + the given header text + data (rawSafetensors, tests/helpers.ts)."""
    text = header_text.encode()
    p = tmp_path / name
    p.write_bytes(struct.pack("<Q", size_override if size_override is not None else len(text)) + text + data)
    return str(p)


def make(we, tmp_path, tensors: dict, metadata=None, name="m.safetensors"):
    p = str(tmp_path / name)
    we.weights.write_safetensors(p, tensors, metadata)
    return p


def test_lists_tensors_with_absolute_offsets(we, tmp_path):  # safetensors.test.ts:8-19
    p = make(we, tmp_path, {"a": ("F8_E4M3", [2, 2], bytes([1, 2, 3, 4])), "b": ("F32", [1], bytes([0, 0, 128, 63]))},
             {"format": "pt"})
    st = we.weights.read_header(p)
    size = (tmp_path / "m.safetensors").stat().st_size
    start = size - 8  # data starts after size + header
    assert st.metadata == {"format": "pt"}
    assert st.tensors["a"] == we.weights.TensorInfo("a", "F8_E4M3", (2, 2), start, 4)
    assert (st.tensors["b"].offset, st.tensors["b"].size) == (start + 4, 4)
    assert list(st.tensors) == ["a", "b"]


def test_reads_one_tensor_without_the_rest(we, tmp_path):  # :21-25
    p = make(we, tmp_path, {"a": ("U8", [2], bytes([7, 8])), "b": ("U8", [3], bytes([9, 10, 11]))})
    st = we.weights.read_header(p)
    assert st.read("b").tolist() == [9, 10, 11]


def test_accepts_a_file_without_tensors(we, tmp_path):  # :27-29
    assert len(we.weights.read_header(make(we, tmp_path, {})).tensors) == 0


@pytest.mark.parametrize("case,message", [
    ("too_small", "too small"),
    ("header_bigger_than_file", "header size"),
    ("header_over_100mb", "header size"),
    ("not_json", "not valid JSON"),
    ("not_object", "not an object"),
    ("unknown_dtype", "unknown dtype"),
    ("bad_shape", "bad shape"),
    ("size_mismatch", "8 bytes"),
    ("past_the_end", "past the end"),
    ("overlap", "overlap"),
    ("bad_offsets", "bad data_offsets"),
    ("deep_nesting", "not valid JSON"),
])
def test_rejects_broken_or_hostile_files(we, tmp_path, case, message):  # :31-55
    files = {
        "too_small": lambda: str((tmp_path / "s").write_bytes(bytes([1, 2])) and tmp_path / "s"),
        "header_bigger_than_file": lambda: raw(tmp_path, "{}", size_override=1000),
        "header_over_100mb": lambda: raw(tmp_path, "{}", size_override=200_000_000),
        "not_json": lambda: raw(tmp_path, "nope"),
        "not_object": lambda: raw(tmp_path, "[1]"),
        "unknown_dtype": lambda: raw(tmp_path, '{"a":{"dtype":"X9","shape":[1],"data_offsets":[0,1]}}', bytes(1)),
        "bad_shape": lambda: raw(tmp_path, '{"a":{"dtype":"U8","shape":[-1],"data_offsets":[0,1]}}', bytes(1)),
        "size_mismatch": lambda: raw(tmp_path, '{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', bytes(4)),
        "past_the_end": lambda: raw(tmp_path, '{"a":{"dtype":"U8","shape":[4],"data_offsets":[0,4]}}', bytes(1)),
        "overlap": lambda: raw(tmp_path, '{"a":{"dtype":"U8","shape":[2],"data_offsets":[0,2]},'
                                         '"b":{"dtype":"U8","shape":[2],"data_offsets":[1,3]}}', bytes(3)),
        "bad_offsets": lambda: raw(tmp_path, '{"a":{"dtype":"U8","shape":[1],"data_offsets":[0]}}', bytes(1)),
        "deep_nesting": lambda: raw(tmp_path, '{"a":' + "[" * 5000 + "]" * 5000 + "}"),
    }
    path = files[case]()
    with pytest.raises(we.weights.SafetensorsError, match=message):
        we.weights.read_header(path)


def test_errors_are_safetensors_errors(we, tmp_path):  # :54
    p = tmp_path / "empty"
    p.write_bytes(b"")
    with pytest.raises(we.weights.SafetensorsError):
        we.weights.read_header(str(p))
    with pytest.raises(OSError):
        we.weights.read_header(str(tmp_path / "missing"))


def test_read_with_a_limit(we, tmp_path):  # :58-64
    st = we.weights.read_header(make(we, tmp_path, {"a": ("U8", [4], bytes([1, 2, 3, 4]))}))
    assert st.read("a", 2).tolist() == [1, 2]


def test_messages_match_the_reference_text(we, tmp_path):
    p = raw(tmp_path, '{"w":{"dtype":"F32","shape":[2],"data_offsets":[0,4]}}', bytes(4))
    with pytest.raises(we.weights.SafetensorsError) as e:
        we.weights.read_header(p)
    assert str(e.value) == "w: has 4 bytes, its shape needs 8 bytes"
    p = raw(tmp_path, "{}", size_override=1000, name="g")
    with pytest.raises(we.weights.SafetensorsError) as e:
        we.weights.read_header(p)
    assert str(e.value) == "Bad header size: 1000"


def test_json_details_follow_json_parse(we, tmp_path):
    """Integral floats are counts (Number.isSafeInteger(2.0)), escapes decode, a repeated key takes the last value."""
    p = raw(tmp_path, '{"a\\u00e9":{"dtype":"U8","shape":[2.0],"data_offsets":[0,2]},'
                      '"b":{"dtype":"X","shape":[1],"data_offsets":[2,3]},"b":{"dtype":"U8","shape":[1],"data_offsets":[2,3]}}',
            bytes(3))
    st = we.weights.read_header(p)
    assert list(st.tensors) == ["aé", "b"] and st.tensors["aé"].shape == (2,)


def test_decoders_equal_the_oracle(we):  # src/weights/fp8.ts:37-53 against oracle/oracle.c
    W = we.weights
    codes = np.arange(256, dtype=np.uint8)
    assert np.array_equal(W.to_float32("F8_E4M3", codes), O.to_float32("F8_E4M3", codes.tobytes()), equal_nan=True)
    assert np.array_equal(W.to_float32("F8_E5M2", codes), O.to_float32("F8_E5M2", codes.tobytes()), equal_nan=True)
    bits = np.random.default_rng(1).integers(0, 65536, 4096, dtype=np.uint16)
    for dt in ("F16", "BF16"):
        assert np.array_equal(W.to_float32(dt, bits.tobytes()), O.to_float32(dt, bits.tobytes()), equal_nan=True)
    f = np.random.default_rng(2).standard_normal(100).astype(np.float32)
    assert np.array_equal(W.to_float32("F32", f.tobytes()), f)
    with pytest.raises(ValueError, match="decode"):
        W.to_float32("I32", bytes(4))


def test_fp8_scaled_pairing_and_block_groups(we, tmp_path):  # src/weights/inspect.ts:9-31
    p = make(we, tmp_path, {
        "blocks.1.attn.wq.weight": ("F8_E4M3", [2, 2], bytes(4)), "blocks.1.attn.wq.weight_scale": ("F32", [], bytes(4)),
        "blocks.0.attn.wq.weight": ("F8_E4M3", [2, 2], bytes(4)), "blocks.0.attn.wq.scale_weight": ("F32", [], bytes(4)),
        "blocks.0.mlp.up.weight": ("F8_E4M3", [2, 2], bytes(4)), "blocks.0.prenorm.scale": ("F32", [2], bytes(8)),
        "txt.layers.0.w.weight": ("BF16", [1], bytes(2)),
    })
    st = we.weights.read_header(p)
    pairs = [(w.name, s.name if s else None) for w, s in we.weights.fp8_weights(st)]
    assert pairs == [("blocks.0.attn.wq.weight", "blocks.0.attn.wq.scale_weight"), ("blocks.0.mlp.up.weight", None),
                     ("blocks.1.attn.wq.weight", "blocks.1.attn.wq.weight_scale")]
    assert we.weights.block_groups(st.tensors) == [("blocks", 2), ("txt.layers", 1)]
