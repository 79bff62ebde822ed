"""Tensor creation (reference: ``core/ops/creation.py:16-608``).

Traced: a scalar ``constant`` broadcast to the shape (``zeros``, ``full``);
``*_like`` ops also fold ``x * 0`` into the result so the argument stays live,
as the reference does; ``constant`` turns an ndarray into a graph constant;
``tril``/``triu`` are ``iota`` compares + ``select``.  Outside a trace the
"cpu" implementations simply call NumPy.
"""

import numpy as np

from nkipy_b200.core.graph import as_graph_tensor, get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef


def _filled(ctx, shape, value, dtype):
    s = as_graph_tensor(ctx, value, dtype)
    if shape:
        s = ctx.build_op("broadcast", [s], tuple(shape), dtype, {"broadcast_dimensions": []})
    return s


def _like(x, value, dtype):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    rdt = np.dtype(dtype) if dtype is not None else np.dtype(t.dtype)
    res = _filled(ctx, tuple(t.shape), value, rdt)
    zero = _filled(ctx, tuple(t.shape), 0.0, t.dtype)
    keep = ctx.build_op("multiply", [t, zero], t.shape, t.dtype)
    if np.dtype(t.dtype) != rdt:
        keep = ctx.build_op("convert", [keep], t.shape, rdt)
    return NKIPyTensorRef(ctx.build_op("add", [res, keep], t.shape, rdt))


zeros = Op("zeros")


@zeros.impl("cpu")
def _zeros_cpu(shape, dtype):
    return np.zeros(shape, dtype=dtype)


@zeros.impl("hlo")
def _zeros(shape, dtype):
    ctx = get_trace_context()
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return NKIPyTensorRef(_filled(ctx, shape, 0.0, np.dtype(dtype)))


full = Op("full")


@full.impl("cpu")
def _full_cpu(shape, fill_value, dtype):
    return np.full(shape, fill_value, dtype=dtype)


@full.impl("hlo")
def _full(shape, fill_value, dtype):
    ctx = get_trace_context()
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return NKIPyTensorRef(_filled(ctx, shape, fill_value, np.dtype(dtype)))


zeros_like = Op("zeros_like")


@zeros_like.impl("cpu")
def _zeros_like_cpu(x, dtype=None):
    return np.zeros_like(x, dtype=dtype)


@zeros_like.impl("hlo")
def _zeros_like(x, dtype=None):
    return _like(x, 0.0, dtype)


ones_like = Op("ones_like")


@ones_like.impl("cpu")
def _ones_like_cpu(x, dtype=None):
    return np.ones_like(x, dtype=dtype)


@ones_like.impl("hlo")
def _ones_like(x, dtype=None):
    return _like(x, 1.0, dtype)


empty_like = Op("empty_like")


@empty_like.impl("cpu")
def _empty_like_cpu(x, dtype=None):
    return np.empty_like(x, dtype=dtype)


@empty_like.impl("hlo")
def _empty_like(x, dtype=None):
    return _like(x, 0.0, dtype)


full_like = Op("full_like")


@full_like.impl("cpu")
def _full_like_cpu(x, fill_value, dtype=None):
    return np.full_like(x, fill_value, dtype=dtype)


@full_like.impl("hlo")
def _full_like(x, fill_value, dtype=None):
    return _like(x, fill_value, dtype)


constant = Op("constant")


@constant.impl("cpu")
def _constant_cpu(value, dtype=None):
    return np.asarray(value, dtype=dtype)


@constant.impl("hlo")
def _constant(value, dtype=None):
    if isinstance(value, NKIPyTensorRef):
        if dtype is not None and value.dtype != np.dtype(dtype):
            from nkipy_b200.core.ops.transform import astype

            return astype(value, dtype)
        return value
    ctx = get_trace_context()
    if dtype is not None:
        dt = np.dtype(dtype)
    elif hasattr(value, "dtype"):
        dt = np.dtype(value.dtype)
    elif isinstance(value, bool):
        dt = np.dtype(np.bool_)
    elif isinstance(value, float):
        dt = np.dtype(np.float32)
    elif isinstance(value, int):
        dt = np.dtype(np.int32)
    else:
        dt = np.asarray(value).dtype
    if isinstance(value, (list, tuple)):
        value = np.asarray(value, dtype=dt)
    return NKIPyTensorRef(as_graph_tensor(ctx, value, dt))


def _triangle(x, k, lower):
    from nkipy_b200.core.ops.elementwise import greater_equal, less_equal, subtract
    from nkipy_b200.core.ops.indexing import where

    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    nd = len(t.shape)
    rows = NKIPyTensorRef(ctx.build_op("iota", [], t.shape, np.int32, {"iota_dimension": nd - 2}))
    cols = NKIPyTensorRef(ctx.build_op("iota", [], t.shape, np.int32, {"iota_dimension": nd - 1}))
    if k != 0:
        cols = subtract(cols, k)
    mask = greater_equal(rows, cols) if lower else less_equal(rows, cols)
    return where(mask, x, 0.0)


tril = Op("tril")


@tril.impl("hlo")
def _tril(x, k=0):
    return _triangle(x, k, True)


triu = Op("triu")


@triu.impl("hlo")
def _triu(x, k=0):
    return _triangle(x, k, False)


diag = Op("diag")


@diag.impl("hlo")
def _diag(v, k=0):
    """1-D -> square matrix with ``v`` on diagonal ``k``; 2-D -> that diagonal."""
    from nkipy_b200.core.ops.elementwise import equal, subtract
    from nkipy_b200.core.ops.indexing import take_along_axis, where
    from nkipy_b200.core.ops.transform import broadcast_to, reshape

    ctx = get_trace_context()
    if len(v.shape) == 1:
        n = v.shape[0] + abs(k)
        rows = NKIPyTensorRef(ctx.build_op("iota", [], (n, n), np.int32, {"iota_dimension": 0}))
        cols = NKIPyTensorRef(ctx.build_op("iota", [], (n, n), np.int32, {"iota_dimension": 1}))
        from nkipy_b200.core.ops.transform import pad as _pad

        padded = _pad(v, (max(0, -k), max(0, k))) if k else v
        # value on row r is padded[col] for k >= 0 (col = r + k), padded[r] for k < 0
        src = reshape(padded, (1, n)) if k >= 0 else reshape(padded, (n, 1))
        full_v = broadcast_to(src, (n, n))
        return where(equal(subtract(cols, k), rows), full_v, 0.0)
    rows_n, cols_n = v.shape
    start_r, start_c = (0, k) if k >= 0 else (-k, 0)
    m = max(0, min(rows_n - start_r, cols_n - start_c))
    idx_r = np.arange(start_r, start_r + m, dtype=np.int32)
    idx_c = np.arange(start_c, start_c + m, dtype=np.int32)
    from nkipy_b200.core.ops.indexing import take

    picked = take(v, idx_r, axis=0)
    return reshape(take_along_axis(picked, idx_c.reshape(m, 1), axis=1), (m,))
