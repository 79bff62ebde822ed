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


# opcodes of the register program (nkipy_b200/csrc/ew_program.cuh)
_LD, _CF, _CI, _IOTA = 1, 2, 3, 4
_UNARY = [20, 21, 22, 23, 24, 25, 26, 27, 28, 29, 30, 31, 32, 33, 34, 60, 61, 62, 63, 100, 101, 102, 103, 104, 105]
_BINARY = [10, 11, 12, 13, 14, 15, 16, 17, 18, 40, 41, 42, 43, 44, 45, 50, 51, 52, 53, 54, 55, 56, 57, 58, 59,
           64, 65, 70, 71, 72, 73, 74, 75, 76, 77, 78, 79, 80, 81, 82, 83]
_SEL = 90


def _random_step(rng):
    """A valid "ew" step: 1-4 inputs of random dtypes over a 1- to 4-axis
    view (dense, broadcast, transposed or reversed), a random program over
    them and an output of a random dtype; the innermost axis a multiple of 4."""
    rank = int(rng.integers(1, 5))
    shape = [int(rng.integers(1, 6)) for _ in range(rank)]
    shape[-1] = 4 * int(rng.integers(1, 9))
    n = int(np.prod(shape))
    dense = [int(np.prod(shape[d + 1:])) for d in range(rank)]
    n_in = int(rng.integers(1, 5))
    ins = []
    for _ in range(n_in):
        kind = rng.integers(0, 4)
        if kind == 0:
            st, off = dense, 0
        elif kind == 1:  # broadcast along random axes
            st = [0 if rng.random() < 0.5 else s for s in dense]
            off = 0
        elif kind == 2:  # reversed innermost axis
            st = dense[:-1] + [-1]
            off = shape[-1] - 1
        else:  # axes permuted (a transposed source)
            perm = list(rng.permutation(rank))
            src = [shape[p] for p in perm]
            sdense = [int(np.prod(src[d + 1:])) for d in range(rank)]
            st = [0] * rank
            for j, p in enumerate(perm):
                st[p] = sdense[j]
            off = 0
        ins.append((int(rng.integers(0, 10)), off, st))
    prog, defined = [], []
    for k in range(n_in):
        prog.append([_LD, k, k, 0, 0, 0, 0, 0])
        defined.append(k)
    nreg = n_in
    if rng.random() < 0.5:
        prog.append([_IOTA, nreg, int(rng.integers(0, rank)), 0, 0, 0, 0, 0])
        defined.append(nreg)
        nreg += 1
    for _ in range(int(rng.integers(3, 12))):
        dst = int(rng.integers(0, min(nreg + 1, 23)))
        a, b, c = (int(rng.choice(defined)) for _ in range(3))
        r = rng.random()
        rnd = int(rng.integers(0, 3)) if rng.random() < 0.3 else 0
        if r < 0.1:
            prog.append([int(rng.choice([_CF, _CI])), dst, 0, 0, 0, int(rng.integers(0, 2 ** 32)), rnd, 0])
        elif r < 0.4:
            prog.append([int(rng.choice(_UNARY)), dst, a, 0, 0, 0, rnd, 0])
        elif r < 0.9:
            bimm = int(rng.random() < 0.3)
            prog.append([int(rng.choice(_BINARY)), dst, a, b, 0, int(rng.integers(0, 2 ** 32)) if bimm else 0, rnd, bimm])
        else:
            prog.append([_SEL, dst, a, b, c, 0, rnd, 0])
        if dst not in defined:
            defined.append(dst)
        nreg = max(nreg, dst + 1)
    out_reg = prog[-1][1]
    ints = [n_in, rank, len(prog), int(rng.integers(0, 10)), out_reg, 0, n] + shape + [0] + dense
    for dt, off, st in ins:
        ints += [dt, off] + list(st)
    for ins_ in prog:
        ints += ins_
    return ints


def test_random_programs_compile():
    """Forty seeded random programs (every opcode, every dtype, broadcast,
    reversed and transposed operands, rounding flags, immediates, iota) all
    compile to a specialised kernel."""
    rng = np.random.default_rng(1234)
    for i in range(40):
        ints = _random_step(rng)
        assert _compile(ints) == 1, (i, ints)
