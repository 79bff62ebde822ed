"""The elementwise chain compiler (``ew_jit.cu``): steps whose innermost axis
has a multiple of 4 elements run on a kernel compiled for that step (NVRTC,
at plan load) instead of the interpreter.  Each test checks through
``nkb_ew_compiler_stats`` that compiled kernels were launched, and compares
with NumPy: exact for integer, compare, select and cast results, 1e-5
relative per element for fp32 arithmetic, one bf16 ulp for bf16 results."""

import ctypes

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200.spike import _nkb
from tests.utils import FP32_RTOL, assert_close, on_device

BF16 = np.dtype(ml_dtypes.bfloat16)
pytestmark = pytest.mark.gpu


def _launched():
    c, f, n = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    _nkb.call("nkb_ew_compiler_stats", ctypes.byref(c), ctypes.byref(f), ctypes.byref(n))
    return n.value


@pytest.mark.parametrize("shape", [(64, 256), (3, 40, 96), (4096 * 8,), (33, 12)])
def test_float_chain_on_compiled_kernel(shape):
    def k(a, b, c):
        t = np.maximum(a * b - c, np.minimum(a, c)) / (1.0 + np.abs(b))
        u = np.where(t >= 0.25, np.sqrt(np.abs(t)) + np.floor(a * 3.0), np.sin(c) * np.cos(b) - np.ceil(t))
        return u * np.tanh(a) + np.log(1.5 + np.abs(c)) - np.sign(b) * np.negative(t)

    rng = np.random.default_rng(61)
    args = [rng.standard_normal(shape, dtype=np.float32) for _ in range(3)]
    before = _launched()
    got = on_device(k, *args)
    assert _launched() > before
    assert_close(got, k(*args), FP32_RTOL)


def test_integer_compare_select_cast_chain_exact():
    def k(x, y, m):
        s = x * 7 + np.abs(y) * y
        r = np.where(m, s, np.maximum(x, y) - np.minimum(x, 3))
        b = (x & 0xFF) ^ (y | 3)
        f = (x.astype(np.float32) * 0.5).astype(np.int32)
        return r + b - f, (x < y) | (s >= 2), np.where(x != y, x, -y)

    rng = np.random.default_rng(62)
    x = rng.integers(-1000, 1000, (48, 128), dtype=np.int32)
    y = rng.integers(-50, 50, (48, 128), dtype=np.int32)
    m = rng.random((48, 128)) < 0.5
    before = _launched()
    got = on_device(k, x, y, m)
    assert _launched() > before
    for g, w in zip(got, k(x, y, m)):
        np.testing.assert_array_equal(np.asarray(g), w)


@pytest.mark.parametrize("dtype", [np.float32, BF16])
def test_transposed_and_broadcast_views(dtype):
    """Operands read through strided views (a transposed input, a row and a
    column broadcast), so the compiled kernel takes its per-axis index
    decomposition and the scalar-load path of non-unit inner strides."""

    def k(a, row, col):
        return np.exp(a.T * 0.5) * row[None, :] + col[:, None]

    rng = np.random.default_rng(63)
    a = rng.standard_normal((96, 40), dtype=np.float32).astype(dtype)
    row = rng.standard_normal((96,), dtype=np.float32).astype(dtype)
    col = rng.standard_normal((40,), dtype=np.float32).astype(dtype)
    before = _launched()
    got = on_device(k, a, row, col)
    assert _launched() > before
    want = k(a, row, col)
    if dtype == BF16:
        # each bf16 node rounds (exp on the device and in NumPy may land one
        # ulp apart): a few ulps of the terms, which can cancel in the sum
        f = np.float32
        terms = np.abs(np.exp(a.T.astype(f) * 0.5) * row.astype(f)[None, :]) + np.abs(col.astype(f)[:, None])
        assert_close(got, want, 2 ** -7, atol=2 ** -6 * terms)
    else:
        assert_close(got, want, FP32_RTOL)


def test_iota_and_bf16_output_exact():
    """tril/triu trace to iota compares on both axes (the row index from the
    kernel's index decomposition, the column from the run's position) and a
    select; one result is converted to bf16 (round to nearest even)."""

    def k(x):
        return np.tril(x, 3).astype(BF16), np.triu(x, -2) * 2.0

    rng = np.random.default_rng(64)
    x = rng.standard_normal((2, 40, 256), dtype=np.float32)
    before = _launched()
    got = on_device(k, x)
    assert _launched() > before
    want = k(x)
    np.testing.assert_array_equal(np.asarray(got[0]).view(np.uint16), np.asarray(want[0]).view(np.uint16))
    np.testing.assert_array_equal(np.asarray(got[1]), want[1])
