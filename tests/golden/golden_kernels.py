"""Kernel bodies whose traced graphs are pinned against the reference tracer.

Both ``make_golden.py`` (run with the reference importable) and
``tests/test_tracer_golden.py`` (run on the committed fixture) use these
exact functions, so the op lists are compared for identical source.
Each entry: (name, function, input factory, kwargs).
"""

import ml_dtypes
import numpy as np

BF16 = np.dtype(ml_dtypes.bfloat16)


def softmax_kernel(x):
    exp_x = np.exp((x - np.max(x, axis=-1, keepdims=True)))
    sum_x = np.sum(exp_x, axis=-1, keepdims=True)
    return exp_x / sum_x


def rmsnorm_residual(x, r, weight):
    h = (x + r).astype(np.float32)
    w = weight.astype(np.float32)
    z = np.mean(np.square(h), axis=-1, keepdims=True)
    return (h / np.sqrt(z + 1e-6) * w).astype(x.dtype)


def matmul_bf16(a, b):
    return a @ b


def bmm(a, b):
    return np.matmul(a, b)


def argmax_last(x):
    return np.argmax(x, axis=-1)


def transpose_copy(x):
    return np.transpose(x, (1, 0, 2))


def take_rows(x, idx):
    return np.take(x, idx, axis=0)


def where_scalar(x, y):
    return np.where(x > y, x, 0.5)


def concat_split(x, y):
    a, b = np.split(np.concatenate([x, y], axis=-1), 2, axis=-1)
    return a * 2.0 + b


def mixed_promotion(x, i):
    return (x * 2 + i).astype(np.float32), i // 3


def mutate_slice(cache, upd):
    cache[:, 2:4] = upd
    return np.sum(cache)


def reductions(x):
    return np.mean(x, axis=0), np.var(x, axis=1), np.max(x)


def rope_like(q, cos, sin):
    half = q.shape[-1] // 2
    q0, q1 = q[..., :half], q[..., half:]
    return np.concatenate([q0 * cos - q1 * sin, q0 * sin + q1 * cos], axis=-1)


def silu_mul(g, u):
    return g * (1 / (1 + np.exp(-g))) * u


def repeat_kv(k):
    return np.repeat(k, 4, axis=2).transpose(0, 2, 1, 3)


def tril_mask(x):
    return np.tril(x) + np.triu(x, k=1) * 0.0


# Op library of the tracer in use, for kernels calling NKIPy ops that are not
# NumPy functions (conv2d / conv3d): set by make_golden.py to the reference's
# ``nkipy.core.ops`` and by the tests to ``nkipy_b200.core.ops``.
OPS = None


def conv2d_bias(x, w, b):
    return OPS.conv2d(x, w, b, stride=(2, 1), padding=(1, 2))


def conv2d_dilated(x, w):
    return OPS.conv2d(x, w, stride=1, padding=2, dilation=2)


def conv3d_bias(x, w, b):
    return OPS.conv3d(x, w, b, stride=1, padding=1)


def _rng(seed):
    return np.random.default_rng(seed)


CASES = [
    ("softmax", softmax_kernel, lambda: (_rng(0).standard_normal((8, 128), dtype=np.float32),), {}),
    (
        "rmsnorm_residual",
        rmsnorm_residual,
        lambda: (
            _rng(1).standard_normal((4, 64), dtype=np.float32),
            _rng(2).standard_normal((4, 64), dtype=np.float32),
            _rng(3).uniform(0.5, 1.5, 64).astype(np.float32),
        ),
        {},
    ),
    ("matmul_bf16", matmul_bf16, lambda: (np.zeros((16, 32), BF16), np.zeros((32, 8), BF16)), {}),
    ("bmm", bmm, lambda: (np.zeros((2, 16, 32), np.float32), np.zeros((2, 32, 8), np.float32)), {}),
    ("argmax_last", argmax_last, lambda: (np.zeros((4, 10), np.float32),), {}),
    ("transpose_copy", transpose_copy, lambda: (np.zeros((2, 3, 4), np.int32),), {}),
    ("take_rows", take_rows, lambda: (np.zeros((10, 6), np.float32), np.array([1, 3, 3], np.int32)), {}),
    ("where_scalar", where_scalar, lambda: (np.zeros((5, 5), np.float32), np.zeros((5,), np.float32)), {}),
    ("concat_split", concat_split, lambda: (np.zeros((3, 4), np.float32), np.zeros((3, 4), np.float32)), {}),
    ("mixed_promotion", mixed_promotion, lambda: (np.zeros((3,), BF16), np.zeros((3,), np.int32)), {}),
    ("mutate_slice", mutate_slice, lambda: (np.zeros((3, 6), np.float32), np.ones((3, 2), np.float32)), {}),
    ("reductions", reductions, lambda: (np.zeros((6, 7), np.float32),), {}),
    (
        "rope_like",
        rope_like,
        lambda: (np.zeros((1, 4, 2, 8), np.float32), np.zeros((1, 4, 1, 4), np.float32), np.zeros((1, 4, 1, 4), np.float32)),
        {},
    ),
    ("silu_mul", silu_mul, lambda: (np.zeros((4, 8), BF16), np.zeros((4, 8), BF16)), {}),
    ("repeat_kv", repeat_kv, lambda: (np.zeros((1, 5, 2, 4), BF16),), {}),
    ("tril_mask", tril_mask, lambda: (np.zeros((2, 5, 5), np.float32),), {}),
    (
        "conv2d_bias",
        conv2d_bias,
        lambda: (np.zeros((2, 3, 9, 11), BF16), np.zeros((4, 3, 3, 2), BF16), np.zeros((4,), BF16)),
        {},
    ),
    ("conv2d_dilated", conv2d_dilated, lambda: (np.zeros((1, 2, 8, 8), np.float32), np.zeros((3, 2, 3, 3), np.float32)), {}),
    (
        "conv3d_bias",
        conv3d_bias,
        lambda: (np.zeros((1, 2, 5, 6, 7), np.float32), np.zeros((3, 2, 2, 3, 2), np.float32), np.zeros((3,), np.float32)),
        {},
    ),
]


def describe(graph):
    """Comparable summary of a traced graph (works on both tracers' graphs)."""

    def norm(v):
        if isinstance(v, np.ndarray):
            return {"ndarray": list(v.shape), "dtype": str(v.dtype), "sum": float(np.asarray(v, dtype=np.float64).sum())}
        if isinstance(v, (list, tuple)):
            return [norm(x) for x in v]
        if isinstance(v, (np.floating, float)):
            return float(v)
        if isinstance(v, (np.integer, int)) and not isinstance(v, bool):
            return int(v)
        return v

    ops = []
    for op in graph.operations:
        ops.append(
            {
                "op": op.op_name,
                "shape": [int(s) for s in op.result_shape],
                "dtype": str(np.dtype(op.result_dtype)),
                "attrs": {k: norm(v) for k, v in sorted(op.attributes.items())},
            }
        )
    return {
        "params": [[p.name, [int(s) for s in p.shape], str(np.dtype(p.dtype))] for p in graph.parameters],
        "ops": ops,
        "results": [[r.name, [int(s) for s in r.shape], str(np.dtype(r.dtype))] for r in graph.results],
        "aliases": [[a.output_index, a.param_index, a.param_name, a.is_user_returned] for a in graph.aliases],
    }
