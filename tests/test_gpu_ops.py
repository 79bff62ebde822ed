"""The remaining op families on the B200 path against the NumPy direct call:
cumsum (reference ``core/ops/reduce.py:317-385``: a product with an
upper-triangular ones matrix, float32 result), pad / roll / tile / repeat /
concatenate (``core/ops/transform.py``).  Layout moves are bit-exact; cumsum is
held to the fp32 bound of a sum, relative to the sum of its terms' magnitudes."""

import ml_dtypes
import numpy as np
import pytest

from tests.utils import FP32_RTOL, assert_close, on_device

BF16 = np.dtype(ml_dtypes.bfloat16)
pytestmark = pytest.mark.gpu


def _exact(got, want):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape and got.dtype == want.dtype, (got.shape, got.dtype, want.shape, want.dtype)
    np.testing.assert_array_equal(got.view(np.uint8), np.ascontiguousarray(want).view(np.uint8))


@pytest.mark.parametrize("shape,axis", [((300, 77), 0), ((64, 1000), -1), ((4, 5, 130), 1), ((513,), 0)])
def test_cumsum_fp32(shape, axis):
    x = np.random.default_rng(30).standard_normal(shape, dtype=np.float32)
    got = on_device(lambda a: np.cumsum(a, axis=axis), x)
    assert_close(got, np.cumsum(x, axis=axis), FP32_RTOL, atol=FP32_RTOL * np.cumsum(np.abs(x), axis=axis))


def test_cumsum_int32_values():
    """The traced cumsum of an integer array is a float32 product (the
    reference's trace promotes it); its values equal NumPy's integer sums."""
    x = np.random.default_rng(31).integers(-50, 50, (5, 40)).astype(np.int32)
    got = on_device(lambda a: np.cumsum(a, axis=1), x)
    np.testing.assert_array_equal(np.asarray(got).astype(np.int64), np.cumsum(x, axis=1))


@pytest.mark.parametrize(
    "shape,pads,value,dtype",
    [((30, 50), ((1, 2), (3, 0)), 0.0, np.float32), ((3, 20, 30), ((0, 0), (2, 2), (1, 1)), 1.5, np.float32),
     ((16, 64), ((4, 4), (0, 8)), 0.0, BF16), ((7, 9), ((2, 0), (0, 3)), 0, np.int32)],
)
def test_pad_exact(shape, pads, value, dtype):
    rng = np.random.default_rng(32)
    x = (rng.integers(-9, 9, shape) if np.dtype(dtype).kind == "i" else rng.standard_normal(shape)).astype(dtype)
    got = on_device(lambda a: np.pad(a, pads, constant_values=value), x)
    _exact(got, np.pad(x, pads, constant_values=value))


@pytest.mark.parametrize("shape,shift,axis,dtype", [((10, 33), 3, 1, np.float32), ((17, 8), -5, 0, BF16),
                                                   ((4, 6, 128), 64, 2, np.float32), ((9, 4), 13, 0, np.int32)])
def test_roll_exact(shape, shift, axis, dtype):
    rng = np.random.default_rng(33)
    x = (rng.integers(-9, 9, shape) if np.dtype(dtype).kind == "i" else rng.standard_normal(shape)).astype(dtype)
    _exact(on_device(lambda a: np.roll(a, shift, axis=axis), x), np.roll(x, shift, axis=axis))


@pytest.mark.parametrize("shape,reps,dtype", [((7, 9), (2, 3), np.float32), ((4, 128), (3, 1), BF16),
                                             ((5,), (4,), np.int32), ((2, 3, 8), (2, 1, 2), np.float32)])
def test_tile_exact(shape, reps, dtype):
    rng = np.random.default_rng(34)
    x = (rng.integers(-9, 9, shape) if np.dtype(dtype).kind == "i" else rng.standard_normal(shape)).astype(dtype)
    _exact(on_device(lambda a: np.tile(a, reps), x), np.tile(x, reps))


@pytest.mark.parametrize("shape,rep,axis,dtype", [((5, 6), 3, 0, np.int32), ((5, 6), 2, 1, BF16),
                                                 ((2, 64, 4, 32), 4, 2, BF16), ((3, 7), 2, 1, np.float32)])
def test_repeat_exact(shape, rep, axis, dtype):
    rng = np.random.default_rng(35)
    x = (rng.integers(-9, 9, shape) if np.dtype(dtype).kind == "i" else rng.standard_normal(shape)).astype(dtype)
    _exact(on_device(lambda a: np.repeat(a, rep, axis=axis), x), np.repeat(x, rep, axis=axis))


@pytest.mark.parametrize("axis", [0, 1])
def test_concatenate_exact(axis):
    rng = np.random.default_rng(36)
    a = rng.standard_normal((4, 5), dtype=np.float32)
    b = rng.standard_normal((4, 7) if axis == 1 else (3, 5), dtype=np.float32)
    _exact(on_device(lambda x, y: np.concatenate([x, y], axis=axis), a, b), np.concatenate([a, b], axis=axis))


def test_integer_matmul_values():
    """An integer product (int32 @ int32 -> int32) on the CUDA-core GEMM,
    accumulated in fp32: exact while every partial sum fits 24 bits."""
    rng = np.random.default_rng(37)
    a = rng.integers(-20, 20, (33, 70)).astype(np.int32)
    b = rng.integers(-20, 20, (70, 45)).astype(np.int32)
    got = on_device(lambda x, y: x @ y, a, b)
    np.testing.assert_array_equal(np.asarray(got).astype(np.int64), a.astype(np.int64) @ b.astype(np.int64))
