"""ctypes binding of the C ABI in include/we_b200.h (libwe_b200.so, built in this directory).

There is no CPU fallback: when the library is missing, or there is no B200, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libwe_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "we_b200.h")

WE_OK, WE_EINVAL, WE_ENOMEM, WE_ECUDA, WE_ENCCL, WE_ETIMEOUT, WE_EUNSUPPORTED, WE_EIO = range(8)
F32, BF16, FP8, INT4G64, F16 = 0, 1, 2, 3, 4
MM_ACCUMULATE, MM_FP8_FAST, MM_FORCE_SIMT, NOALLOC_SYNC = 1, 2, 4, 8
NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024
STREAM_HOST_PINNED = 1
COMM_ID_BYTES = 128
REDUCE_SUM, REDUCE_MAX = 0, 1
ROPE_INTERLEAVED, ROPE_HALF = 0, 1
EW = {"swiglu": 0, "sigmoid_gate": 1, "gated_add": 2, "add_bias": 3, "gelu_tanh": 4, "add": 5, "silu": 6}
ACTS = {None: 0, "none": 0, "gelu_tanh": 1, "silu": 2}
AUX_OPS = {None: 0, "none": 0, "sigmoid_gate": 1, "swiglu": 2}

DTYPES = {"f32": F32, "bf16": BF16, "fp8": FP8, "int4": INT4G64, "f16": F16}
DTYPE_BYTES = {F32: 4, BF16: 2, FP8: 1, F16: 2}


class WeError(RuntimeError):
    """A non-OK status from the library; `code` is the WE_* status."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class Stats(C.Structure):
    _fields_ = [("created", C.c_uint64), ("reused", C.c_uint64), ("created_bytes", C.c_uint64),
                ("launches", C.c_uint64), ("tc_gemms", C.c_uint64), ("simt_gemms", C.c_uint64)]


class Epilogue(C.Structure):
    _fields_ = [("act", C.c_int32), ("aux_op", C.c_int32), ("aux_dtype", C.c_int32), ("aux", C.c_void_p),
                ("gate", C.c_void_p)]


class MatmulDesc(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("m", "n", "k", "x_stride", "w_stride", "y_stride", "x_offset", "w_offset",
                                         "y_offset", "k_split")] + [
        ("scale", C.c_float), ("chan_scale", C.c_void_p), ("group_scale", C.c_void_p), ("bias", C.c_void_p),
        ("x_dtype", C.c_int32), ("w_dtype", C.c_int32), ("y_dtype", C.c_int32), ("flags", C.c_uint32),
        ("epi", Epilogue)]


GEMM_MAX_SEGMENTS = 32


class GemmFp8Desc(C.Structure):
    _fields_ = [("m", C.c_int64), ("n", C.c_int64), ("k", C.c_int64), ("x_hi", C.c_void_p), ("x_lo", C.c_void_p),
                ("row_scale", C.c_void_p), ("w", C.c_void_p), ("scale", C.c_float), ("chan_scale", C.c_void_p),
                ("bias", C.c_void_p), ("y", C.c_void_p), ("y_stride", C.c_int64), ("y_dtype", C.c_int32),
                ("flags", C.c_uint32), ("epi", Epilogue), ("y_parts", C.c_void_p * 3), ("part_n", C.c_int64 * 3),
                ("w2", C.c_void_p), ("scale2", C.c_float), ("chan_scale2", C.c_void_p), ("bias2", C.c_void_p),
                ("gate2", C.c_void_p), ("nseg", C.c_int32), ("row_end", C.c_int64 * GEMM_MAX_SEGMENTS),
                ("row_set", C.c_int32 * GEMM_MAX_SEGMENTS), ("peer_dst", C.c_void_p * 8), ("peer_world", C.c_int32),
                ("peer_part", C.c_int32), ("peer_row0", C.c_int64)]


class LinearDesc(C.Structure):
    pass


LinearDesc._fields_ = [("weight", C.c_void_p), ("dtype", C.c_int32), ("scale", C.c_float), ("chan_scale", C.c_void_p),
                       ("group_scale", C.c_void_p), ("n", C.c_int64), ("k", C.c_int64), ("bias", C.c_void_p),
                       ("lora_down", C.POINTER(LinearDesc)), ("lora_up", C.POINTER(LinearDesc))]


class StTensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_char_p), ("ndim", C.c_int32), ("shape", C.c_int64 * 8),
                ("offset", C.c_int64), ("size", C.c_int64)]


class PeerCopy(C.Structure):
    _fields_ = [("src", C.c_void_p), ("rows", C.c_int64), ("chunk_bytes", C.c_int64), ("src_row_stride", C.c_int64),
                ("src_peer_stride", C.c_int64), ("dst_offset", C.c_int64), ("dst_row_stride", C.c_int64),
                ("dst_rank_stride", C.c_int64)]


PEER_MAX = 8
PEER_HANDLE_BYTES = 128


class ModDesc(C.Structure):
    _fields_ = [("scale", C.c_void_p), ("shift", C.c_void_p)]


class RopeDesc(C.Structure):
    _fields_ = [("cos", C.c_void_p), ("sin", C.c_void_p), ("pairs", C.c_int64), ("tokens", C.c_int64)]


_P = C.c_void_p
_I64 = C.c_int64
_SIGS = {
    "we_init": (C.c_int, [C.c_int, C.c_uint32, C.POINTER(C.c_void_p)]),
    "we_destroy": (C.c_int, [_P]),
    "we_last_error": (C.c_char_p, [_P]),
    "we_set_stream": (C.c_int, [_P, _P]),
    "we_get_stream": (_P, [_P]),
    "we_sync": (C.c_int, [_P]),
    "we_device_error": (C.c_int, [_P, C.POINTER(C.c_uint32)]),
    "we_num_sms": (C.c_int, [_P]),
    "we_buffer": (C.c_int, [_P, C.c_size_t, _P, C.POINTER(C.c_void_p)]),
    "we_write": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "we_read": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "we_copy": (C.c_int, [_P, _P, C.c_size_t, _P, C.c_size_t, C.c_size_t]),
    "we_mark": (C.c_size_t, [_P]),
    "we_release": (C.c_int, [_P, C.c_size_t, C.POINTER(C.c_void_p), C.c_size_t]),
    "we_free": (C.c_int, [_P, _P]),
    "we_get_stats": (C.c_int, [_P, C.POINTER(Stats)]),
    "we_matmul": (C.c_int, [_P, C.POINTER(MatmulDesc), _P, _P, _P]),
    "we_matmul_check": (C.c_int, [_P, C.POINTER(MatmulDesc)]),
    "we_gemm_fp8": (C.c_int, [_P, C.POINTER(GemmFp8Desc)]),
    "we_ksplit_for": (_I64, [_I64, _I64, _I64]),
    "we_linear_forward": (C.c_int, [_P, _P, C.c_int32, C.POINTER(LinearDesc), _I64, C.c_int32, C.c_uint32,
                                    C.POINTER(C.c_void_p)]),
    "we_linear_host": (C.c_int, [_P, _P, C.c_int32, C.POINTER(LinearDesc), _I64, C.c_int32, C.c_uint32, _P, _I64]),
    "we_no_mod": (C.c_int, [_P, _I64, C.POINTER(ModDesc)]),
    "we_norm": (C.c_int, [_P, _P, C.c_int32, _P, _I64, _I64, C.POINTER(ModDesc), C.c_float, C.c_float, C.c_int32,
                          C.POINTER(C.c_void_p)]),
    "we_rotate": (C.c_int, [_P, _P, C.c_int32, _I64, C.POINTER(RopeDesc), C.c_int32, C.c_int32,
                            C.POINTER(C.c_void_p)]),
    "we_rmsnorm": (C.c_int, [_P, _P, C.c_int32, _P, _P, _P, _I64, _I64, C.c_float, C.c_float, _P, C.c_int32]),
    "we_rope_apply": (C.c_int, [_P, _P, C.c_int32, _P, _P, _I64, _I64, _I64, C.c_int32, _P, C.c_int32]),
    "we_qknorm_rope": (C.c_int, [_P, _P, C.c_int32, _P, C.c_float, C.c_float, _P, _P, _I64, _I64, _I64, C.c_int32, _P,
                                 C.c_int32]),
    "we_rope_tables": (_I64, [_P, _I64, C.c_int32, _P, C.c_double, _P, _P]),
    "we_positions": (C.c_int, [_I64, _I64, _I64, _P]),
    "we_unpack_fp8": (C.c_int, [_P, _P, _I64, C.c_float, _P]),
    "we_unpack_fp8_bf16": (C.c_int, [_P, _P, _I64, _P]),
    "we_unpack_int4": (C.c_int, [_P, _P, _P, _I64, _I64, _P]),
    "we_quantize_fp8": (C.c_int, [_P, _P, C.c_int32, _I64, _I64, C.c_int32, _P, _P]),
    "we_quantize_int4": (C.c_int, [_P, _P, C.c_int32, _I64, _I64, _P, _P]),
    "we_quantize_act": (C.c_int, [_P, _P, C.c_int32, _I64, _I64, _I64, C.c_int32, _P, _P, _P]),
    "we_elementwise": (C.c_int, [_P, C.c_int32, _P, _P, _P, _I64, _I64, C.c_int32, _P, C.c_int32]),
    "we_ew": (C.c_int, [_P, C.c_int32, _P, _P, _P, _I64, _I64, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "we_norm_split": (C.c_int, [_P, _P, C.c_int32, _P, _P, _P, _I64, _I64, C.c_float, C.c_float, C.c_int32, _P, _P,
                                _P]),
    "we_capture_begin": (C.c_int, [_P]),
    "we_capture_end": (C.c_int, [_P, C.POINTER(C.c_void_p)]),
    "we_graph_launch": (C.c_int, [_P, _P]),
    "we_graph_destroy": (C.c_int, [_P, _P]),
    "we_add_norm_split": (C.c_int, [_P, _P, _P, _P, _P, _P, _P, _I64, _I64, C.c_float, C.c_float, C.c_int32, _P, _P,
                                    _P]),
    "we_head_groups": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, C.c_int32]),
    "we_patchify": (C.c_int, [_P, _P, C.c_int32, _I64, _I64, _I64, _P, C.c_int32]),
    "we_unpatchify": (C.c_int, [_P, _P, C.c_int32, _I64, _I64, _I64, _P, C.c_int32]),
    "we_attention": (C.c_int, [_P, _P, _P, _P, C.c_int32, _I64, _I64, _I64, _I64, C.c_int32, _P, C.c_int32]),
    "we_attend": (C.c_int, [_P, _P, _P, _P, C.c_int32, _I64, _I64, _I64, _I64, C.c_int32, C.c_int32,
                            C.POINTER(C.c_void_p)]),
    "we_streamer_create": (C.c_int, [_P, C.POINTER(C.c_void_p), C.POINTER(C.c_size_t), C.c_int32, C.c_int32,
                                     C.c_uint32, C.POINTER(C.c_void_p)]),
    "we_streamer_acquire": (C.c_int, [_P, C.c_int32, C.POINTER(C.c_void_p)]),
    "we_streamer_release": (C.c_int, [_P, C.c_int32]),
    "we_streamer_stats": (C.c_int, [_P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "we_streamer_destroy": (C.c_int, [_P]),
    "we_st_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_size_t]),
    "we_st_count": (_I64, [_P]),
    "we_st_tensor_at": (C.c_int, [_P, _I64, C.POINTER(StTensor)]),
    "we_st_find": (C.c_int, [_P, C.c_char_p, C.POINTER(StTensor)]),
    "we_st_metadata_count": (_I64, [_P]),
    "we_st_metadata_at": (C.c_int, [_P, _I64, C.POINTER(C.c_char_p), C.POINTER(C.c_char_p)]),
    "we_st_read": (C.c_int, [_P, C.c_char_p, _P, _I64]),
    "we_st_upload": (C.c_int, [_P, _P, C.c_char_p, _P]),
    "we_st_close": (None, [_P]),
    "we_peer_create": (C.c_int, [_P, C.c_int32, C.c_int32, C.c_size_t, C.POINTER(C.c_void_p)]),
    "we_peer_export": (C.c_int, [_P, _P]),
    "we_peer_open": (C.c_int, [_P, _P]),
    "we_peer_region": (C.c_void_p, [_P]),
    "we_peer_exchange": (C.c_int, [_P, _P, _P, C.c_int32, C.c_uint64]),
    "we_peer_remote": (C.c_void_p, [_P, C.c_int32]),
    "we_qknorm_rope_peers": (C.c_int, [_P, _P, _P, C.c_float, C.c_float, _P, _P, _I64, _I64, C.c_int32, _P, C.c_int32,
                                       _I64]),
    "we_peer_destroy": (C.c_int, [_P]),
    "we_matmul_fp8_noalloc": (C.c_int, [_P, _P, _I64, _I64, _I64, _P, _I64, C.c_float, _P, _P, _P, _I64, C.c_int32,
                                        C.c_uint32, C.c_char_p, C.c_size_t]),
    "we_copy_2d": (C.c_int, [_P, _P, C.c_size_t, _P, C.c_size_t, C.c_size_t, C.c_size_t]),
    "we_comm_unique_id": (C.c_int, [_P]),
    "we_comm_init": (C.c_int, [_P, C.c_int32, C.c_int32, _P, C.c_uint64, C.POINTER(C.c_void_p)]),
    "we_comm_destroy": (C.c_int, [_P]),
    "we_comm_abort": (C.c_int, [_P]),
    "we_comm_rank": (C.c_int, [_P, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "we_comm_last_error": (C.c_char_p, [_P]),
    "we_all_gather": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "we_reduce_scatter": (C.c_int, [_P, _P, _P, C.c_size_t, C.c_int32]),
    "we_all_reduce": (C.c_int, [_P, _P, _P, C.c_size_t, C.c_int32, C.c_int32]),
    "we_all_to_all": (C.c_int, [_P, _P, _P, C.c_size_t]),
    "we_comm_barrier": (C.c_int, [_P]),
    "we_comm_wait": (C.c_int, [_P]),
}

_lib = None


def header_symbols() -> list[str]:
    """Every entry point declared in include/we_b200.h."""
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(we_[a-z0-9_]+)\s*\(", text)))


def lib() -> C.CDLL:
    """The loaded library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"web-engine B200 library not built ({LIB_PATH}); run __graft_entry__.build()")
        lib_ = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib_, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib_
    return _lib


def check(ctx, rc: int) -> None:
    if rc != WE_OK:
        msg = lib().we_last_error(ctx)
        raise WeError(rc, (msg.decode() if msg else "") or f"web-engine error {rc}")
