"""Spec-driven kernel suite, in the form of the reference's
``tests/integration/test_kernels.py:19-93`` and ``test_kernels_fuzz.py:42-119``:
every ``kernel_specs`` entry of ``tests/kernels/*.py`` is run with its default
inputs and with fuzzed shapes and dtypes inside its ``ShapeSpec`` /
``TypeSpec``, on the B200 through the C ABI, against the NumPy direct call.
Without a GPU the kernels are traced and planned only (the reference's
``trace_and_compile`` path when no device is present).

Tolerance: the reference's device bar (``tests/utils.py:19-20``, rtol = atol =
1e-2) with the absolute part scaled by the output's magnitude when bf16 or fp16
is involved (a low-precision product's error is relative to its terms); fp32
kernels are held to 1e-4 (the reference's CPU bar), scaled the same way."""

import glob
import importlib
import os
import random

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200.core.specs import KernelSpec, ScalarInputSpec, TensorInputSpec

HERE = os.path.dirname(os.path.abspath(__file__))
LOW = (np.dtype(ml_dtypes.bfloat16), np.dtype(np.float16))


def collect_kernel_specs():
    """``kernel_specs`` of every module under tests/kernels, keyed 'file:i'."""
    out = {}
    for path in sorted(glob.glob(os.path.join(HERE, "kernels", "*.py"))):
        name = os.path.splitext(os.path.basename(path))[0]
        if name.startswith("_"):
            continue
        mod = importlib.import_module(f"tests.kernels.{name}")
        for i, spec in enumerate(getattr(mod, "kernel_specs", [])):
            assert isinstance(spec, KernelSpec)
            out[f"{name}:{i}"] = spec
    return out


SPECS = collect_kernel_specs()


def _value(shape, dtype, rng):
    dt = np.dtype(dtype)
    if dt.kind in "iu":
        return rng.integers(0, 8, shape).astype(dt)
    if dt == np.bool_:
        return rng.random(shape) < 0.5
    return rng.standard_normal(shape).astype(np.float32).astype(dt)


def make_inputs(spec: KernelSpec, seed: int, fuzz: bool):
    """Default shapes and dtypes, or (fuzz) one random size per distinct
    (min, max) range of the spec -- inputs that declare the same range get the
    same size, which keeps them consistent -- and a random allowed dtype per
    input.  Inputs with a ``default_value`` keep it."""
    rng = np.random.default_rng(seed)
    pick = random.Random(seed)
    sizes = {}
    args = []
    for inp in spec.inputs:
        if inp.default_value is not None:
            args.append(inp.default_value)
            continue
        if isinstance(inp, ScalarInputSpec):
            args.append(inp.dtype_spec.default)
            continue
        assert isinstance(inp, TensorInputSpec)
        if not fuzz:
            shape, dtype = inp.shape_spec.default, inp.dtype_spec.default
        else:
            shape = []
            for d in inp.shape_spec.dims:
                if isinstance(d, int):
                    shape.append(d)
                else:
                    lo, hi = d if isinstance(d, tuple) else (None, None)
                    key = (lo, hi)
                    if key not in sizes:
                        sizes[key] = pick.randint(lo or 1, hi or 64)
                    shape.append(sizes[key])
            dtype = pick.choice(inp.dtype_spec.allowed)
        args.append(_value(tuple(shape), dtype, rng))
    return args


def _check(got, want, low):
    got, want = np.asarray(got), np.asarray(want)
    assert got.shape == want.shape, (got.shape, want.shape)
    if want.dtype.kind in "iub":
        np.testing.assert_array_equal(got, want)
        return
    g, w = got.astype(np.float32), want.astype(np.float32)
    tol = 1e-2 if low else 1e-4
    peak = max(1.0, float(np.max(np.abs(w)))) if w.size else 1.0
    np.testing.assert_allclose(g, w, rtol=tol, atol=tol * peak)


def _run_and_check(spec, args):
    from tests.utils import on_device

    low = any(isinstance(a, np.ndarray) and a.dtype in LOW for a in args)
    want = spec.function(*[a.copy() if isinstance(a, np.ndarray) else a for a in args])
    got = on_device(spec.function, *[a.copy() if isinstance(a, np.ndarray) else a for a in args])
    if isinstance(want, tuple):
        assert isinstance(got, tuple) and len(got) == len(want)
        for g, w in zip(got, want):
            _check(g, w, low)
    else:
        _check(got, want, low)


def test_specs_collected():
    assert len(SPECS) >= 10


@pytest.mark.parametrize("key", sorted(SPECS))
def test_kernel_spec_traces_and_plans(key):
    """Every spec traces and plans on CPU (no device): the default and two fuzzed inputs."""
    import tempfile

    from nkipy_b200.core.trace import NKIPyKernel
    from nkipy_b200.runtime import compile as C

    spec = SPECS[key]
    for seed, fuzz in ((0, False), (1, True), (2, True)):
        args = make_inputs(spec, seed, fuzz)
        k = NKIPyKernel.trace(spec.function)
        k.specialize(*args)
        C.compile_to_plan(k, tempfile.mkdtemp(), name="spec", world=1, use_cached_if_exists=False)


@pytest.mark.gpu
@pytest.mark.parametrize("key", sorted(SPECS))
def test_kernel_spec_default(key):
    _run_and_check(SPECS[key], make_inputs(SPECS[key], 0, False))


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [11, 12, 13])
@pytest.mark.parametrize("key", sorted(SPECS))
def test_kernel_spec_fuzz(key, seed):
    _run_and_check(SPECS[key], make_inputs(SPECS[key], seed, True))
