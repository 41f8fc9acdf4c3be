"""The restatement of numpy's float32 exp and row sum that the sampling kernels use, pinned
against numpy itself on the CPU.

The reference samples decisions in numpy float32 (cardgym/rl/ppo.py:75-94). The kernels
reproduce numpy's exp (its SIMD routine on AVX2/AVX-512 hosts) and its pairwise last-axis sum
(card_playing_gym_b200/csrc/numpy_math.cuh); oracle/numpy_f32.c states the same two
functions in C. These tests hold the C statement to np.exp and np.sum bit for bit, so the GPU
tests that compare the kernels with numpy test the kernels.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import numpy_f32

try:
    from numpy._core._multiarray_umath import __cpu_features__ as _FEATURES
except ImportError:  # pragma: no cover - numpy layout of other versions
    _FEATURES = {}

needs_simd_exp = pytest.mark.skipif(not (_FEATURES.get("AVX2") and _FEATURES.get("FMA3")),
                                    reason="numpy uses libm's expf without AVX2/FMA3")


@needs_simd_exp
def test_exp_matches_numpy_on_sampled_float32():
    rng = np.random.default_rng(11)
    parts = [
        -rng.random(4_000_000, dtype=np.float32) * 104,          # the whole shifted-logit range
        -rng.random(4_000_000, dtype=np.float32) * 2,            # where softmax mass lives
        -rng.random(1_000_000, dtype=np.float32) * 1e-3,         # next to zero
        -(87 + rng.random(1_000_000, dtype=np.float32) * 17),    # subnormal and zero results
        rng.random(1_000_000, dtype=np.float32) * 88.7,          # positive arguments
    ]
    special = np.array([0.0, -0.0, -np.inf, np.inf, np.nan, 88.72283935546875, 88.7228317, -103.97208404541015625,
                        -103.972076, -87.33654, -1e-45, np.finfo(np.float32).tiny], dtype=np.float32)
    x = np.concatenate(parts + [special]).astype(np.float32)
    got, want = numpy_f32.expf(x), np.exp(x)
    same = (got.view(np.uint32) == want.view(np.uint32)) | (np.isnan(got) & np.isnan(want))
    assert same.all(), f"{(~same).sum()} differences, first at x={x[~same][:4]}"


@needs_simd_exp
def test_exp_matches_numpy_on_every_float32_near_zero():
    """Every float32 in [-2^-4, 0] and the 2^22 below -1 (exhaustive slices)."""

    bits = np.concatenate([np.arange(0x80000000, 0xBD800001, dtype=np.uint64)[::7],
                           np.arange(0xBF800000, 0xBFC00000, dtype=np.uint64)]).astype(np.uint32)
    x = bits.view(np.float32)
    assert np.array_equal(numpy_f32.expf(x).view(np.uint32), np.exp(x).view(np.uint32))


@pytest.mark.parametrize("width", [1, 3, 7, 8, 9, 11, 16, 52, 64, 127, 128, 129, 200, 255, 256, 300, 489, 512])
def test_row_sum_matches_numpy(width):
    rng = np.random.default_rng(width)
    rows = 4000
    scale = rng.choice([1e-6, 1e-3, 1.0, 1e3], size=(rows, width)).astype(np.float32)
    a = rng.random((rows, width), dtype=np.float32) * scale
    a[rng.random((rows, width)) < 0.6] = 0.0
    assert np.array_equal(numpy_f32.row_sums(a), a.sum(axis=-1, keepdims=True)[:, 0])
