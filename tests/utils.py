"""Shared helpers (reference tests/utils.py:17-95): run a kernel on the B200
and compare with the NumPy direct call."""

import numpy as np

from nkipy_b200.core.trace import NKIPyKernel

# tolerances of the benchmark definition
FP32_RTOL = 1e-5
BF16_RTOL = 2e-2


def on_device(kernel_fn, *args, **kwargs):
    from nkipy_b200.runtime import baremetal_run_traced_kernel

    return baremetal_run_traced_kernel(NKIPyKernel.trace(kernel_fn), *args, **kwargs)


def f32(x):
    return np.asarray(x).astype(np.float32)


def rel_err(got, want):
    got, want = f32(got), f32(want)
    return float(np.max(np.abs(got - want)) / max(1e-30, float(np.max(np.abs(want)))))


def assert_close(got, want, rtol, atol=None):
    got, want = f32(got), f32(want)
    assert got.shape == want.shape, (got.shape, want.shape)
    if atol is None:
        atol = rtol * max(1e-30, float(np.max(np.abs(want)))) if want.size else 0.0
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)
