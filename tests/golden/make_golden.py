"""Writes the golden vectors that pin the CPU oracle (tests/golden/golden.json).

Run in a container that has PyTorch and the reference checkout:

    python tests/golden/make_golden.py /path/to/web-engine

Sources of truth, all independent of oracle/oracle.c:
  * PyTorch itself: float8_e4m3fn / float8_e5m2 / bfloat16 / float16 decoding and encoding,
    and ``torch.manual_seed(s); torch.randn(n)``, which the reference's src/model/noise.ts
    restates and its tests/fixtures/torch-randn.json records;
  * the reference's own fixture tests/fixtures/torch-randn.json (read as data);
  * numpy float64 restatements of the reference tests' matmul / rmsnorm / rope formulas
    (tests/gpu/matmul.test.ts:26-35, tests/gpu/rmsnorm.test.ts:10-20, src/kernels/rope.ts:20-36)
    on the reference tests' LCG inputs (tests/gpu/matmul.test.ts:10-23);
  * torch restatements of this build's own quantisation conventions (per-channel fp8,
    int4 group-64, two-term e4m3 activation split), so the C oracle is checked against a
    second implementation.
The output is small (a few hundred KB) and is committed; the tests never need torch or
the reference checkout.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import sys

import numpy as np
import torch

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.json")


def lcg(seed):
    state = [seed & 0xFFFFFFFF]

    def r():
        state[0] = (state[0] * 1664525 + 1013904223) & 0xFFFFFFFF
        return state[0] / 2 ** 32

    return r


def torch_decode(codes, dtype, view_int):
    t = torch.tensor(codes, dtype=view_int).view(dtype)
    return [None if math.isnan(v) else v for v in t.float().tolist()]


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def matmul_cases():
    """tests/gpu/matmul.test.ts:14-23 data() + :26-35 reference(), restated with numpy float64."""
    e4 = torch.arange(256, dtype=torch.int32).to(torch.uint8).view(torch.float8_e4m3fn).double().numpy()
    cases = []
    for (m, n, k, seed, scale) in [(1, 1, 4, 1, 0.002), (37, 70, 100, 1, 0.002), (64, 64, 64, 1, 0.002),
                                   (130, 65, 36, 1, 0.002), (200, 260, 84, 1, 0.002),
                                   (8, 1536, 6144, 7, 0.0018833705689758062)]:
        r = lcg(seed)
        x = np.array([r() * 2 - 1 for _ in range(m * k)], dtype=np.float32)
        w = []
        for _ in range(n * k):
            b = math.floor(r() * 256)
            w.append(b - 1 if (b & 0x7F) == 0x7F else b)
        w = np.array(w, dtype=np.uint8)
        y = (x.astype(np.float64).reshape(m, k) @ e4[w].reshape(n, k).T) * scale
        pick = [0, (m * n) // 3, (m * n) // 2, m * n - 1]
        cases.append({"m": m, "n": n, "k": k, "seed": seed, "scale": scale, "x_sha256": digest(x),
                      "w_sha256": digest(w), "y_at": {str(i): float(y.ravel()[i]) for i in pick},
                      "y_sum": float(y.sum()), "y_abs_sum": float(np.abs(y).sum())})
    return cases


def rmsnorm_cases():
    """tests/gpu/rmsnorm.test.ts:5-8 rng (centred) and :10-20 reference(), numpy float64."""
    def rng(seed):
        base = lcg(seed)
        return lambda: base() - 0.5

    out = []
    for (seed, rows, d, offset, mod) in [(1, 3, 6144, 1.0, True), (2, 100, 128, 0.0, False), (3, 5, 37, 1.0, False)]:
        r = rng(seed)
        if mod:
            x = np.array([r() * 8 for _ in range(rows * d)], dtype=np.float32)
            w = np.array([r() * 0.2 for _ in range(d)], dtype=np.float32)
            sc = np.array([r() * 2 for _ in range(d)], dtype=np.float32)
            sh = np.array([r() * 2 for _ in range(d)], dtype=np.float32)
        else:
            x = np.array([r() * 2 for _ in range(rows * d)], dtype=np.float32)
            w = np.array([r() * 2 for _ in range(d)], dtype=np.float32)
            sc = np.zeros(d, np.float32)
            sh = np.zeros(d, np.float32)
        xd = x.astype(np.float64).reshape(rows, d)
        inv = 1 / np.sqrt((xd ** 2).sum(1) / d + 1e-5)
        y = xd * inv[:, None] * (offset + w.astype(np.float64)) * (1 + sc.astype(np.float64)) + sh
        out.append({"seed": seed, "rows": rows, "d": d, "offset": offset, "mod": mod, "x_sha256": digest(x),
                    "y_at": {str(i): float(y.ravel()[i]) for i in (0, y.size // 2, y.size - 1)},
                    "y_sum": float(y.sum())})
    return out


def rope_tables_np(pos, axes, theta):
    pairs = sum(a // 2 for a in axes)
    cos = np.zeros((len(pos), pairs), np.float32)
    sin = np.zeros((len(pos), pairs), np.float32)
    for t, p in enumerate(pos):
        pair = 0
        for a, dim in enumerate(axes):
            for j in range(dim // 2):
                ang = p[a] * theta ** (-(2 * j) / dim)
                cos[t, pair] = math.cos(ang)
                sin[t, pair] = math.sin(ang)
                pair += 1
    return cos, sin


def main(ref_root: str) -> None:
    g = {"note": "Golden vectors for the CPU oracle; made by tests/golden/make_golden.py with torch "
                 + torch.__version__ + ". Do not edit by hand."}
    codes = list(range(256))
    g["e4m3"] = torch_decode(codes, torch.float8_e4m3fn, torch.uint8)
    g["e5m2"] = torch_decode(codes, torch.float8_e5m2, torch.uint8)
    f16codes = [0x0000, 0x8000, 0x3C00, 0xC000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0x7C00, 0xFC00, 0x3555, 0x5A3C]
    g["f16"] = {"codes": f16codes, "values": torch_decode([c - 65536 if c > 32767 else c for c in f16codes],
                                                        torch.float16, torch.int16)}
    bfcodes = [0x3F80, 0xC000, 0x0001, 0x7F7F, 0x4049, 0xBF00]
    g["bf16"] = {"codes": bfcodes, "values": torch_decode([c - 65536 if c > 32767 else c for c in bfcodes],
                                                         torch.bfloat16, torch.int16)}

    # encoders: RNE (ties included); torch's e4m3 cast is used only inside the finite range
    gen = torch.Generator().manual_seed(1234)
    vals = torch.cat([torch.randn(2000, generator=gen) * 40, torch.randn(500, generator=gen) * 0.01,
                      torch.tensor([0.0, -0.0, 448.0, -448.0, 2 ** -9, 2 ** -10, 3 * 2 ** -10, 1.0625, 1.1875,
                                    240.0, 232.0, 0.015625, 0.0146484375, 449.0, 463.0])])
    vals = vals[vals.abs() < 464]
    g["e4m3_encode"] = {"in": vals.tolist(), "out": vals.to(torch.float8_e4m3fn).view(torch.uint8).tolist()}
    bvals = torch.cat([torch.randn(1000, generator=gen) * 3, torch.tensor([1.00390625, 1.01171875, -2.00781250])])
    g["bf16_encode"] = {"in": bvals.tolist(), "out": [v & 0xFFFF for v in
                                                      bvals.to(torch.bfloat16).view(torch.int16).tolist()]}
    hvals = torch.cat([torch.randn(1000, generator=gen) * 5, torch.randn(200, generator=gen) * 1e-5,
                       torch.tensor([70000.0, 65504.0, 65520.0, 1.00048828125])])
    g["f16_encode"] = {"in": hvals.tolist(), "out": [int(v) for v in
                                                     hvals.numpy().astype(np.float16).view(np.uint16).tolist()]}

    # torch randn: the reference fixture's cases, regenerated with real torch
    fixture = json.load(open(os.path.join(ref_root, "tests/fixtures/torch-randn.json")))
    cases = []
    for c in fixture["cases"]:
        torch.manual_seed(c["seed"])
        a = torch.randn(c["n"])
        for i, v in c["values"].items():
            assert abs(a[int(i)].item() - v) < 1e-5, (c["n"], c["seed"], i)
        cases.append({"n": c["n"], "seed": c["seed"], "values": {i: a[int(i)].item() for i in c["values"]}})
    for (n, seed) in [(6, 0), (3, 42), (16, 0), (100, 7), (17, 3), (3072, 0)]:
        torch.manual_seed(seed)
        a = torch.randn(n)
        pick = sorted(set([0, 1, n // 2, n - 1] + list(range(max(0, n - 16), n))))
        cases.append({"n": n, "seed": seed, "values": {str(i): a[i].item() for i in pick}})
    g["torch_randn"] = cases

    g["matmul"] = matmul_cases()
    g["rmsnorm"] = rmsnorm_cases()

    # rope tables (src/kernels/rope.ts:20-36) on reference test positions
    rp = []
    for (pos, axes, theta) in [([[0, 3, 5]], [32, 48, 48], 1000.0), ([[0, 1, 2], [0, 7, 9]], [16, 56, 56], 1e4),
                               ([[0], [1], [5], [40]], [128], 5e6)]:
        c, s = rope_tables_np(pos, axes, theta)
        rp.append({"pos": pos, "axes": axes, "theta": theta, "cos": c.ravel().tolist(), "sin": s.ravel().tolist()})
    g["rope_tables"] = rp

    # this build's quantisers, restated in torch
    r = lcg(11)  # inputs from the reference tests' LCG: bit-identical in numpy and torch
    w = torch.from_numpy(np.array([(r() * 2 - 1) * 0.02 for _ in range(64 * 256)], np.float32).reshape(64, 256))
    amax = w.abs().amax(1)
    s = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (w / s[:, None]).to(torch.float8_e4m3fn).view(torch.uint8)
    g["quant_fp8_channel"] = {"seed": 11, "n": 64, "k": 256, "std": 0.02, "w_sha256": digest(w.numpy()),
                              "scales": s.tolist(), "q_sha256": digest(q.numpy())}
    sg = (w.view(64, 4, 64).abs().amax(2) / 7.0).to(torch.float16)
    qi = torch.round(w.view(64, 4, 64) / sg.float()[:, :, None]).clamp(-8, 7).to(torch.int32).view(64, 256)
    nib = (qi & 0xF).to(torch.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).contiguous()
    operand = (qi.view(64, 4, 64).float() * sg.float()[:, :, None]).to(torch.bfloat16).float().view(64, 256)
    g["quant_int4_g64"] = {"seed": 11, "n": 64, "k": 256, "std": 0.02,
                           "scales": sg.view(torch.int16).flatten().tolist(), "packed_sha256": digest(packed.numpy()),
                           "operand_sha256": digest(operand.numpy())}
    r = lcg(5)
    xa = torch.from_numpy(np.array([(r() * 2 - 1) * 3 for _ in range(4 * 512)], np.float32).reshape(4, 512))
    xa = xa.to(torch.bfloat16).float()
    xa[1] *= 300.0
    xa[2] *= 1e-3
    xa[3] = 0
    splits = []
    for row in xa:
        amax = row.abs().max().item()
        e = 0
        if amax > 0:
            e = math.ceil(math.log2(amax / 448.0))
            while amax * 2.0 ** (-(e - 1)) <= 448.0:
                e -= 1
            while amax * 2.0 ** (-e) > 448.0:
                e += 1
        v = row * 2.0 ** (-e)
        hi = v.to(torch.float8_e4m3fn)
        lo = (v - hi.float()).to(torch.float8_e4m3fn)
        splits.append({"e": e, "hi_sha256": digest(hi.view(torch.uint8).numpy()),
                       "lo_sha256": digest(lo.view(torch.uint8).numpy()),
                       "exact": bool(((hi.float() + lo.float()) * 2.0 ** e == row).all())})
    g["act_split"] = {"seed": 5, "rows": 4, "k": 512, "scale_rows": [1.0, 300.0, 1e-3, 0.0], "rows_out": splits}

    json.dump(g, open(OUT, "w"), indent=0)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference checkout>")
    main(sys.argv[1])
