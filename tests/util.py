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
