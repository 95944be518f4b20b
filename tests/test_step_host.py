"""The step driver's host parts against the reference's own tests (no GPU): the oracle restatements of
timestepEmbedding / patchify / unpatchify (tests/transformer.test.ts), sigmas / eulerStep / gaussian
(tests/sampler.test.ts), and the package's host functions against the oracle."""
import math

import numpy as np
import pytest

from oracle import oracle as O


def test_timestep_embedding():  # tests/transformer.test.ts:5-18
    e = O.timestep_embedding(0.7)
    assert e.size == 256
    assert abs(e[0] - math.cos(700)) < 5e-6 and abs(e[128] - math.sin(700)) < 5e-6
    assert abs(e[127] - math.cos(700 * 10000 ** (-127 / 128))) < 5e-6
    z = O.timestep_embedding(0)
    assert np.array_equal(z[:128], np.ones(128)) and np.array_equal(z[128:], np.zeros(128))


def test_patchify_cases():  # tests/transformer.test.ts:21-52
    h, w = 4, 6
    lat = np.arange(16 * h * w, dtype=np.float32)
    t = O.patchify(lat, h, w)
    assert t.size == (h // 2) * (w // 2) * 64
    assert t[(1 * 3 + 2) * 64 + 3 * 4 + 1 * 2 + 0] == lat[(3 * h + 3) * w + 4]
    lat = np.sin(np.arange(16 * 8 * 8)).astype(np.float32)
    assert np.array_equal(O.unpatchify(O.patchify(lat, 8, 8), 8, 8), lat)
    h, w = 3, 5
    lat = np.arange(16 * h * w, dtype=np.float32)
    t = O.patchify(lat, h, w)
    assert t.size == 2 * 3 * 64
    assert t[(0 * 3 + 2) * 64 + 5 * 4 + 0 * 2 + 1] == lat[(5 * h + 0) * w + 0]
    assert t[(1 * 3 + 1) * 64 + 5 * 4 + 1 * 2 + 0] == lat[(5 * h + 0) * w + 2]
    lat = np.cos(np.arange(16 * 5 * 7)).astype(np.float32)
    assert np.array_equal(O.unpatchify(O.patchify(lat, 5, 7), 5, 7), lat)


def test_sigmas_and_euler():  # tests/sampler.test.ts:4-24
    s = O.sigmas()
    assert len(s) == 9 and abs(s[0] - 1) < 1e-10 and s[8] == 0
    assert all(s[i] < s[i - 1] for i in range(1, 9))
    e = math.exp(1.15)
    assert abs(s[7] - e / (e + 8 - 1)) < 1e-10
    assert O.sigmas(1) == [1.0, 0.0]
    assert O.euler_step([1, 2], [4, -2], 1, 0.75).tolist() == [0, 2.5]


def test_gaussian():  # tests/sampler.test.ts:26-35
    a = O.gaussian(20000, 42)
    assert np.array_equal(a[:5], O.gaussian(5, 42))
    assert abs(a.mean()) < 0.03 and abs(a.std() - 1) < 0.03


def test_package_host_functions_equal_the_oracle(we):
    T = we.transformer
    for t in (0.0, 0.3, 0.7, 1.0):
        assert np.array_equal(T.timestep_embedding(t), O.timestep_embedding(t))
    for steps in (1, 4, 8):
        assert np.allclose(T.sigmas(steps), O.sigmas(steps), rtol=0, atol=1e-15)
    assert np.array_equal(T.gaussian(1001, 7), O.gaussian(1001, 7))
    assert T.patch_grid(3, 5) == O.patch_grid(3, 5) == (2, 3)


def test_step_flops_match_the_benchmark_arithmetic(we):
    """Config 4: 57 blocks of 4608 tokens -> 59.5 TF of block linears and 14.9 TF of attention."""
    T = we.transformer
    f = T.step_flops(T.StepConfig(), 512, 4096)
    blk = we.blocks.block_flops(T.FLUX_BLOCK, 4608)
    assert blk["linear"] == 2 * 4608 * (4 * 3072 ** 2 + 2 * 3072 * 12288)
    assert abs(57 * blk["linear"] / 1e12 - 59.5) < 0.05 and abs(f["attention"] / 1e12 - 14.87) < 0.05


def test_block_config_checks_its_shapes(we):
    B = we.blocks.BlockConfig
    B(hidden=256, mlp=1024, heads=2, kv_heads=1, head_dim=128)
    with pytest.raises(ValueError, match="must equal hidden"):
        B(hidden=256, mlp=1024, heads=4, kv_heads=2, head_dim=128)
    with pytest.raises(ValueError, match="multiple of kvHeads"):
        B(hidden=384, mlp=1024, heads=3, kv_heads=2, head_dim=128)
