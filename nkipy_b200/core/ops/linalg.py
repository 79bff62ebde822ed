"""Contractions (reference: ``core/ops/linalg.py:15-316``).

``matmul`` follows NumPy: 1-D operands are promoted to 2-D by ``reshape`` and
the added axis removed afterwards; batch axes broadcast (``broadcast`` nodes)
before one ``dot`` node whose attributes name the contracting and batch
dimensions.  ``dot`` outer-products the non-contracted axes.  The result
dtype is the promoted operand dtype (bf16 @ bf16 -> bf16).
"""

import numpy as np

from nkipy_b200.core.graph import broadcast_to_shape, find_common_type, get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef


def _dot_node(ctx, a, b, shape, dtype, lc, rc, lb, rb):
    return ctx.build_op(
        "dot",
        [a, b],
        shape,
        dtype,
        {
            "lhs_contracting_dimensions": lc,
            "rhs_contracting_dimensions": rc,
            "lhs_batch_dimensions": lb,
            "rhs_batch_dimensions": rb,
        },
    )


matmul = Op("matmul")


@matmul.impl("hlo")
def _matmul(x, y, out=None, dtype=None):
    ctx = get_trace_context()
    rdt = find_common_type(x, y)
    a = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    b = y.backend_tensor if isinstance(y, NKIPyTensorRef) else y
    assert len(a.shape) >= 1 and len(b.shape) >= 1, "matmul requires at least 1D arrays"
    drop_l = drop_r = False
    if len(a.shape) == 1 and len(b.shape) == 1:
        assert a.shape[0] == b.shape[0], "Incompatible shapes for dot product"
        r = _dot_node(ctx, a, b, (), rdt, [0], [0], [], [])
        return NKIPyTensorRef(r)
    if len(a.shape) == 1:
        a = ctx.build_op("reshape", [a], (1, a.shape[0]), a.dtype)
        drop_l = True
    if len(b.shape) == 1:
        b = ctx.build_op("reshape", [b], (b.shape[0], 1), b.dtype)
        drop_r = True
    assert a.shape[-1] == b.shape[-2], "Incompatible shapes for matmul"
    batch = tuple(np.broadcast_shapes(tuple(a.shape[:-2]), tuple(b.shape[:-2])))
    ta = batch + tuple(a.shape[-2:])
    tb = batch + tuple(b.shape[-2:])
    if tuple(a.shape) != ta:
        a = broadcast_to_shape(ctx, a, ta)
    if tuple(b.shape) != tb:
        b = broadcast_to_shape(ctx, b, tb)
    shape = batch + (a.shape[-2], b.shape[-1])
    bd = list(range(len(batch)))
    r = _dot_node(ctx, a, b, shape, rdt, [len(ta) - 1], [len(tb) - 2], bd, list(bd))
    if drop_l or drop_r:
        fs = list(shape)
        if drop_l:
            fs.pop(-2)
        if drop_r:
            fs.pop(-1)
        r = ctx.build_op("reshape", [r], tuple(fs), rdt)
    return NKIPyTensorRef(r)


dot = Op("dot")


@dot.impl("hlo")
def _dot(x, y, out=None):
    ctx = get_trace_context()
    rdt = find_common_type(x, y)
    a = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    b = y.backend_tensor if isinstance(y, NKIPyTensorRef) else y
    lc = [len(a.shape) - 1]
    rc = [max(0, len(b.shape) - 2)]
    assert a.shape[lc[0]] == b.shape[rc[0]], f"shapes {a.shape} and {b.shape} not aligned"
    shape = tuple(s for i, s in enumerate(a.shape) if i not in lc) + tuple(
        s for i, s in enumerate(b.shape) if i not in rc
    )
    return NKIPyTensorRef(_dot_node(ctx, a, b, shape, rdt, lc, rc, [], []))


norm = Op("norm")


@norm.impl("hlo")
def _norm(x, ord=None, axis=None, keepdims=False):
    from nkipy_b200.core.ops.elementwise import multiply, sqrt
    from nkipy_b200.core.ops.reduce import sum as _sum

    if ord is not None and ord != "fro":
        raise NotImplementedError(f"Only L2/Frobenius norm is supported (ord=None or 'fro'), got ord={ord}")
    if ord == "fro":
        if len(x.shape) < 2 or (axis is not None and (not isinstance(axis, (list, tuple)) or len(axis) < 2)):
            raise ValueError("Invalid norm order 'fro' for vectors")
    return sqrt(_sum(multiply(x, x), axis=axis, keepdims=keepdims))


outer = Op("outer")


@outer.impl("hlo")
def _outer(a, b, out=None):
    from nkipy_b200.core.ops.elementwise import multiply
    from nkipy_b200.core.ops.transform import reshape

    return multiply(reshape(a, (-1, 1)), reshape(b, (1, -1)))


trace = Op("trace")


@trace.impl("hlo")
def _trace(a, offset=0, axis1=0, axis2=1, dtype=None):
    from nkipy_b200.core.ops.elementwise import equal, subtract
    from nkipy_b200.core.ops.indexing import where
    from nkipy_b200.core.ops.reduce import sum as _sum
    from nkipy_b200.core.ops.transform import astype

    ctx = get_trace_context()
    t = a.backend_tensor if isinstance(a, NKIPyTensorRef) else a
    nd = len(t.shape)
    axis1 = axis1 + nd if axis1 < 0 else axis1
    axis2 = axis2 + nd if axis2 < 0 else axis2
    rows = NKIPyTensorRef(ctx.build_op("iota", [], t.shape, np.dtype(np.int32), {"iota_dimension": axis1}))
    cols = NKIPyTensorRef(ctx.build_op("iota", [], t.shape, np.dtype(np.int32), {"iota_dimension": axis2}))
    if offset != 0:
        cols = subtract(cols, offset)
    r = where(equal(rows, cols), a, 0.0)
    for ax in sorted([axis1, axis2], reverse=True):
        r = _sum(r, axis=ax)
    if dtype is not None:
        r = astype(r, np.dtype(dtype))
    return r
