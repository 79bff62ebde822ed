"""Reductions (reference: ``core/ops/reduce.py:14-486``).

``sum``/``max``/``min``/``prod`` become one ``reduce`` node (operand + scalar
init constant, attributes ``dimensions`` and ``computation``) followed by a
``reshape`` when ``keepdims``.  ``mean``/``var``/``std`` are sums and divides;
``argmax``/``argmin`` are max -> compare -> float ``iota`` -> select -> min ->
``convert`` to int32 (first occurrence wins); ``cumsum`` is a matmul with an
upper-triangular ones matrix.
"""

import builtins

import numpy as np

from nkipy_b200.core.graph import as_graph_tensor, get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef

_INIT = {"add": 0.0, "maximum": float("-inf"), "minimum": float("inf"), "multiply": 1.0}


def _norm_axes(axis, ndim):
    if axis is None:
        return tuple(range(ndim))
    if isinstance(axis, (list, tuple)):
        return tuple(a + ndim if a < 0 else a for a in axis)
    return (axis + ndim if axis < 0 else axis,)


def _reduce(computation, x, axis=None, keepdims=False):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    dims = _norm_axes(axis, len(t.shape))
    out_shape = tuple(s for i, s in enumerate(t.shape) if i not in dims)
    init = as_graph_tensor(ctx, _INIT[computation], t.dtype)
    r = ctx.build_op(
        "reduce", [t, init], out_shape, t.dtype, {"dimensions": list(dims), "computation": computation}
    )
    if keepdims:
        kshape = tuple(1 if i in dims else s for i, s in enumerate(t.shape))
        r = ctx.build_op("reshape", [r], kshape, t.dtype)
    return NKIPyTensorRef(r)


def _count(shape, axis):
    if axis is None:
        return int(np.prod(shape))
    return int(np.prod([shape[a] for a in _norm_axes(axis, len(shape))]))


def _make_reduce(name, computation):
    op = Op(name)

    @op.impl("hlo")
    def _impl(x, axis=None, out=None, dtype=None, keepdims=False, initial=None):
        return _reduce(computation, x, axis=axis, keepdims=keepdims)

    return op


sum = _make_reduce("sum", "add")  # noqa: A001
max = _make_reduce("max", "maximum")  # noqa: A001
min = _make_reduce("min", "minimum")  # noqa: A001
prod = _make_reduce("prod", "multiply")

mean = Op("mean")


@mean.impl("hlo")
def _mean(x, axis=None, out=None, dtype=None, keepdims=False, initial=None):
    from nkipy_b200.core.ops.elementwise import divide
    from nkipy_b200.core.ops.transform import astype

    if dtype is not None:
        x = astype(x, np.dtype(dtype))
    s = sum(x, axis=axis, keepdims=keepdims)
    return divide(s, float(_count(x.shape, axis)))


any = Op("any")  # noqa: A001


@any.impl("hlo")
def _any(x, axis=None, out=None, dtype=None, keepdims=False):
    from nkipy_b200.core.ops.elementwise import not_equal
    from nkipy_b200.core.ops.transform import astype

    nz = astype(not_equal(x, 0), np.dtype(np.int32))
    return not_equal(sum(nz, axis=axis, keepdims=keepdims), 0)


var = Op("var")


@var.impl("hlo")
def _var(x, axis=None, out=None, dtype=None, keepdims=False, ddof=0):
    from nkipy_b200.core.ops.elementwise import divide, multiply, subtract
    from nkipy_b200.core.ops.transform import astype

    if dtype is not None:
        x = astype(x, np.dtype(dtype))
    m = mean(x, axis=axis, keepdims=True)
    c = subtract(x, m)
    ss = sum(multiply(c, c), axis=axis, keepdims=keepdims)
    n = _count(x.shape, axis) - ddof
    return divide(ss, float(n if n > 0 else 0))


std = Op("std")


@std.impl("hlo")
def _std(x, axis=None, out=None, dtype=None, keepdims=False, ddof=0):
    from nkipy_b200.core.ops.elementwise import sqrt

    return sqrt(var(x, axis=axis, dtype=dtype, keepdims=keepdims, ddof=ddof))


def _arg_extreme(x, axis, keepdims, extreme):
    from nkipy_b200.core.ops.elementwise import equal
    from nkipy_b200.core.ops.indexing import where
    from nkipy_b200.core.ops.transform import astype, reshape

    ctx = get_trace_context()
    ref = x if isinstance(x, NKIPyTensorRef) else NKIPyTensorRef(x)
    orig_shape, orig_axis = ref.shape, axis
    if axis is None:
        ref = reshape(ref, (int(np.prod(ref.shape)),))
        axis = 0
    if axis < 0:
        axis += ref.ndim
    best = extreme(ref, axis=axis, keepdims=True)
    mask = equal(ref, best)
    iota = NKIPyTensorRef(
        ctx.build_op("iota", [], ref.shape, np.dtype(np.float32), {"iota_dimension": axis})
    )
    picked = where(mask, iota, float(ref.shape[axis] + 1))
    res = astype(min(picked, axis=axis), np.dtype(np.int32))
    if keepdims:
        if orig_axis is not None:
            ks = list(orig_shape)
            ks[orig_axis] = 1
        else:
            ks = [1] * len(orig_shape)
        res = reshape(res, tuple(ks))
    return res


argmax = Op("argmax")


@argmax.impl("hlo")
def _argmax(x, axis=None, out=None, keepdims=False):
    return _arg_extreme(x, axis, keepdims, max)


argmin = Op("argmin")


@argmin.impl("hlo")
def _argmin(x, axis=None, out=None, keepdims=False):
    return _arg_extreme(x, axis, keepdims, min)


cumsum = Op("cumsum")


@cumsum.impl("hlo")
def _cumsum(x, axis=None, dtype=None):
    from nkipy_b200.core.ops.creation import constant
    from nkipy_b200.core.ops.linalg import matmul
    from nkipy_b200.core.ops.transform import astype, reshape, transpose

    shape = x.shape
    nd = len(shape)
    if axis is None:
        x = reshape(x, (int(np.prod(shape)),))
        shape, nd, axis = (int(np.prod(shape)),), 1, 0
    elif axis < 0:
        axis += nd
    n = shape[axis]
    tri = constant(np.triu(np.ones((n, n), dtype=np.float32)))
    if nd == 1:
        res = reshape(matmul(reshape(x, (1, n)), tri), (n,))
    elif axis == nd - 1:
        rows = int(np.prod(shape[:-1]))
        res = reshape(matmul(reshape(x, (rows, n)), tri), shape)
    else:
        perm = list(range(nd))
        perm[axis], perm[-1] = perm[-1], perm[axis]
        xt = transpose(x, axes=perm)
        tshape = tuple(shape[p] for p in perm)
        rows = int(np.prod(tshape[:-1]))
        res = transpose(reshape(matmul(reshape(xt, (rows, n)), tri), tshape), axes=perm)
    if dtype is not None and res.dtype != np.dtype(dtype):
        res = astype(res, np.dtype(dtype))
    return res


count_nonzero = Op("count_nonzero")


@count_nonzero.impl("hlo")
def _count_nonzero(x, axis=None, keepdims=False):
    from nkipy_b200.core.ops.elementwise import not_equal
    from nkipy_b200.core.ops.transform import astype

    return sum(astype(not_equal(x, 0), np.dtype(np.int32)), axis=axis, keepdims=keepdims)


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("builtins", "np")]
