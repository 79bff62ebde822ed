"""The elementwise chain compiler on the host: kernels traced here, planned,
and each planned ``ew`` step's specialised kernel compiled with NVRTC through
``nkb_ew_compile_step`` (no GPU is used).  Steps whose innermost axis has a
multiple of 4 elements must be taken and compile; the others are left to the
interpreter.  Skipped where NVRTC itself is not installed."""

import ctypes
import ctypes.util
import tempfile

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200.core.trace import NKIPyKernel
from nkipy_b200.runtime.compile import compile_to_plan, specialize
from nkipy_b200.spike import _nkb

BF16 = np.dtype(ml_dtypes.bfloat16)


def _have_nvrtc():
    for name in ("libnvrtc.so.12", "libnvrtc.so"):
        try:
            ctypes.CDLL(name)
            return True
        except OSError:
            pass
    return False


pytestmark = pytest.mark.skipif(not _have_nvrtc(), reason="NVRTC not installed")


def _ew_steps(fn, *args):
    k = NKIPyKernel.trace(fn)
    specialize(k, args, {})
    path = compile_to_plan(k, tempfile.mkdtemp(), name="ew_cpu")
    steps = []
    for line in open(path).read().splitlines():
        tok = line.split()
        if len(tok) > 2 and tok[0] == "step" and tok[1] == "ew":
            nb = int(tok[2])
            rest = tok[3 + 2 * nb:]
            ni = int(rest[0])
            steps.append([int(v) for v in rest[1:1 + ni]])
    return steps


def _compile(ints):
    arr = (ctypes.c_int64 * len(ints))(*ints)
    taken = ctypes.c_int()
    _nkb.call("nkb_ew_compile_step", arr, len(ints), ctypes.byref(taken))
    return taken.value


def _inner(ints):
    rank = ints[1]
    return ints[7 + rank - 1]


def _float_chain(a, b, c):
    t = np.maximum(a * b - c, np.minimum(a, c)) / (1.0 + np.abs(b))
    u = np.where(t >= 0.25, np.sqrt(np.abs(t)) + np.floor(a * 3.0), np.sin(c) * np.cos(b) - np.ceil(t))
    return u * np.tanh(a) + np.log(1.5 + np.abs(c)) - np.sign(b) * np.negative(t)


def _int_chain(x, y, m):
    s = x * 7 + np.abs(y) * y
    r = np.where(m, s, np.maximum(x, y) - np.minimum(x, 3))
    return r + ((x & 0xFF) ^ (y | 3)) - (x.astype(np.float32) * 0.5).astype(np.int32), (x < y) | (s >= 2)


def _views(a, row, col):
    return np.exp(a.T * 0.5) * row[None, :] + col[:, None]


def _tril(x):
    return np.tril(x, 3).astype(BF16), np.triu(x, -2) * 2.0


@pytest.mark.parametrize("case", ["float", "float_odd", "int", "views_f32", "views_bf16", "tril"])
def test_planned_chains_compile(case):
    rng = np.random.default_rng(5)
    f32 = lambda *s: rng.standard_normal(s, dtype=np.float32)  # noqa: E731
    if case == "float":
        steps = _ew_steps(_float_chain, f32(64, 256), f32(64, 256), f32(64, 256))
    elif case == "float_odd":
        steps = _ew_steps(_float_chain, f32(37, 65), f32(37, 65), f32(37, 65))
    elif case == "int":
        x = rng.integers(-9, 9, (48, 128), dtype=np.int32)
        steps = _ew_steps(_int_chain, x, x + 1, rng.random((48, 128)) < 0.5)
    elif case == "views_f32":
        steps = _ew_steps(_views, f32(96, 40), f32(96), f32(40))
    elif case == "views_bf16":
        steps = _ew_steps(_views, f32(96, 40).astype(BF16), f32(96).astype(BF16), f32(40).astype(BF16))
    else:
        steps = _ew_steps(_tril, f32(2, 40, 256))
    assert steps
    for ints in steps:
        want = 1 if _inner(ints) % 4 == 0 else 0
        assert _compile(ints) == want, ints[:12]


def test_compile_step_rejects_bad_parameters():
    assert _nkb.lib().nkb_ew_compile_step(None, 0, None) != 0
    taken = ctypes.c_int(7)
    bad = (ctypes.c_int64 * 3)(1, 2, 3)
    assert _nkb.lib().nkb_ew_compile_step(bad, 3, ctypes.byref(taken)) != 0
    assert taken.value == 0
