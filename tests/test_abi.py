"""CPU checks of the C-ABI library: it loads, exports every declared entry point, and its host-only
functions (no GPU needed) agree with the oracle. No kernel is launched here."""
import ctypes as C
import glob
import os
import subprocess

import numpy as np
import pytest

from oracle import oracle as O


def test_library_exports_every_declared_symbol(we):
    lib = we._lib.lib()
    declared = we._lib.header_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", we._lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T we_" in line}
    assert set(declared) <= exported
    assert set(we._lib._SIGS) == set(declared)  # the ctypes binding covers the whole header


def test_library_targets_sm100a_only(we):
    out = subprocess.run(["/usr/local/cuda/bin/cuobjdump", "--list-elf", we._lib.LIB_PATH], capture_output=True,
                         text=True).stdout
    assert "sm_100a" in out and "sm_90" not in out


def test_ksplit_for_matches_reference(we):  # tests/gpu/matmul.test.ts:151-156
    assert we.k_split_for(1088, 64, 6144) == 24
    assert we.k_split_for(4160, 64, 16384) == 8
    assert we.k_split_for(4160, 6144, 6144) == 1
    assert we.k_split_for(5, 12, 16) == 1
    for m, n, k in [(1, 1, 1), (256, 3072, 3072), (4608, 12288, 3072), (8, 1536, 6144), (300, 16, 4096)]:
        assert we.k_split_for(m, n, k) == O.ksplit_for(m, n, k)


def test_matmul_params_refuses_unaligned_layouts(we):  # tests/gpu/matmul.test.ts:68-72
    with pytest.raises(ValueError, match="K must be a multiple of 4"):
        we.kernels.matmul_params(1, 1, 6, 1.0)
    with pytest.raises(ValueError, match="xStride"):
        we.kernels.matmul_params(1, 1, 4, 1.0, x_stride=6)
    with pytest.raises(ValueError, match="wOffset"):
        we.kernels.matmul_params(1, 1, 4, 1.0, w_offset=2)


def test_matmul_check_in_the_library_uses_the_reference_messages(we):
    lib = we._lib.lib()
    d = we.kernels.matmul_params(1, 1, 4, 1.0)
    d.k = 6
    d.x_stride = d.w_stride = 0
    # we_matmul_check with a NULL context still returns the status (the message needs a context)
    assert lib.we_matmul_check(None, C.byref(d)) == we._lib.WE_EINVAL
    d.k = 8
    assert lib.we_matmul_check(None, C.byref(d)) == we._lib.WE_OK
    d.w_dtype = we._lib.INT4G64
    assert lib.we_matmul_check(None, C.byref(d)) == we._lib.WE_EINVAL  # K % 64 and group scales


def test_rope_tables_and_positions_match_oracle(we):
    pos = we.kernels.positions(2, 3, 4)
    assert pos.tolist() == O.positions(2, 3, 4).tolist()
    for axes, theta in [((32, 48, 48), 1000.0), ((16, 56, 56), 1e4)]:
        cos, sin, pairs = we.kernels.rope_tables(pos, axes, theta)
        oc, osn, op = O.rope_tables(pos, axes, theta)
        assert pairs == op and np.array_equal(cos, oc) and np.array_equal(sin, osn)
    cos, sin, pairs = we.kernels.rope_tables([[0], [1], [5], [40]], (128,), 5e6)
    oc, osn, _ = O.rope_tables([[0], [1], [5], [40]], (128,), 5e6)
    assert np.array_equal(cos, oc) and np.array_equal(sin, osn)
    with pytest.raises(ValueError, match="even"):
        we.kernels.rope_tables([[0, 0, 0]], (31, 48, 49))


@pytest.mark.skipif(bool(glob.glob("/dev/nvidia[0-9]*")), reason="only meaningful without a GPU")
def test_without_a_gpu_the_library_fails_loudly(we):
    with pytest.raises(we._lib.WeError):
        we.Graph(0)


def test_noalloc_refuses_bad_arguments_before_touching_the_gpu(we):
    """we_matmul_fp8_noalloc checks its arguments before any CUDA call, so these refusals need no GPU: negative
    sizes, row strides shorter than a row (or negative), K not a multiple of 16, an unaligned w."""
    lib = we._lib.lib()
    dummy = C.c_void_p(256)  # never dereferenced: every case below is refused first

    def call(m, k, x_stride, n, y_stride, w=dummy):
        err = C.create_string_buffer(200)
        rc = lib.we_matmul_fp8_noalloc(None, dummy, m, k, x_stride, w, n, 1.0, None, None, dummy, y_stride,
                                       we._lib.DTYPES["bf16"], 0, err, 200)
        return rc, err.value.decode()

    for args, words in [((-1, 64, 0, 16, 0), "negative"), ((4, 64, 32, 16, 0), "x_stride"),
                        ((4, 64, -64, 16, 0), "x_stride"), ((4, 64, 0, 16, 8), "y_stride"),
                        ((4, 64, 0, 16, -1), "y_stride"), ((4, 40, 0, 16, 0), "multiple of 16")]:
        rc, msg = call(*args)
        assert rc == we._lib.WE_EINVAL and words in msg, (args, msg)
    rc, msg = call(4, 64, 0, 16, 0, w=C.c_void_p(257))
    assert rc == we._lib.WE_EINVAL and "aligned" in msg
