"""Shared helpers (reference tests/utils.py:17-95): run a kernel on the B200
and compare with the NumPy direct call."""

import numpy as np

from nkipy_b200.core.trace import NKIPyKernel

# tolerances of the benchmark definition
FP32_RTOL = 1e-5
BF16_RTOL = 2e-2
# absolute floor of the fp32 comparison, per unit of the output's scale
# (max(1, max|want|)): about one ulp of a value of that size, so an element
# whose exact value is near zero, where a relative bound means nothing, is
# held to the rounding of the terms it was computed from and every other
# element to its own 1e-5 relative bound
FP32_ATOL_SCALE = 1e-7


def on_device(kernel_fn, *args, **kwargs):
    from nkipy_b200.runtime import baremetal_run_traced_kernel

    return baremetal_run_traced_kernel(NKIPyKernel.trace(kernel_fn), *args, **kwargs)


def f32(x):
    return np.asarray(x).astype(np.float32)


def rel_err(got, want):
    got, want = f32(got), f32(want)
    return float(np.max(np.abs(got - want)) / max(1e-30, float(np.max(np.abs(want)))))


def assert_close(got, want, rtol, atol=None):
    """Elementwise ``|got - want| <= atol + rtol * |want|``.

    fp32 work (``rtol <= FP32_RTOL``): ``atol`` defaults to
    ``FP32_ATOL_SCALE * max(1, max|want|)``, so the bound is relative per
    element.  bf16 matmul paths (``rtol = BF16_RTOL``): ``atol`` defaults to
    ``rtol * max|want|`` -- a product rounded to bf16 carries an error
    relative to the size of the dot product's terms, not of its (possibly
    cancelled) sum.  Reductions whose result may cancel pass an explicit
    ``atol`` from the sum of the magnitudes of their terms
    (``sum_abs_atol``)."""
    got, want = f32(got), f32(want)
    assert got.shape == want.shape, (got.shape, want.shape)
    if atol is None:
        peak = float(np.max(np.abs(want))) if want.size else 0.0
        if rtol <= FP32_RTOL:
            atol = FP32_ATOL_SCALE * max(1.0, peak)
        else:
            atol = rtol * max(1e-30, peak)
    if np.ndim(atol) == 0:
        np.testing.assert_allclose(got, want, rtol=rtol, atol=float(atol))
        return
    bound = np.broadcast_to(f32(atol), want.shape) + rtol * np.abs(want)
    bad = ~(np.abs(got - want) <= bound)
    if np.any(bad):
        i = np.unravel_index(int(np.argmax(bad)), want.shape)
        raise AssertionError(f"{int(bad.sum())} of {want.size} elements outside the per-element bound; first at {i}: "
                             f"got {got[i]!r}, want {want[i]!r}, bound {bound[i]!r}")


def sum_abs_atol(x, axis, rtol=FP32_RTOL):
    """Per-output absolute bound of a floating-point sum over ``axis``:
    ``rtol * sum|x|`` (the classical bound of a sum's rounding error is a
    multiple of the unit roundoff times the sum of the magnitudes of its
    terms, whatever the order of the additions)."""
    return rtol * np.sum(np.abs(f32(x)), axis=axis)
