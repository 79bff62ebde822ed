"""Selection, gather and scatter (reference: ``core/ops/indexing.py:17-862``).

* ``where`` -> ``select`` (a non-bool condition is first compared ``!= 0``);
* ``take`` -> ``gather`` with XLA dimension numbers (one collapsed axis);
* ``take_along_axis`` -> per-axis index grids concatenated into one index
  vector per element, then a point ``gather``;
* ``static_slice`` -> ``slice`` (+ ``reshape`` to drop integer-indexed axes);
* ``dynamic_update_slice`` -> ``dynamic-update-slice`` with scalar int32
  ``constant`` start indices;
* ``scatter_along_axis`` / ``scatter_strided`` / ``put_along_axis`` ->
  ``scatter`` with ``update_computation = "assign"``.
"""

import itertools

import numpy as np

from nkipy_b200.core.graph import (
    TraceOp,
    as_graph_tensor,
    broadcast_to_shape,
    find_common_type,
    get_trace_context,
)
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef


def _const(ctx, arr, dtype=None):
    arr = np.asarray(arr)
    if dtype is not None:
        arr = arr.astype(dtype)
    return ctx.module.add_operation(TraceOp("constant", [], arr.shape, arr.dtype, {"value": arr}))


where = Op("where")


@where.impl("hlo")
def _where(condition, x, y):
    ctx = get_trace_context()
    out_dt = find_common_type(x, y)
    if isinstance(condition, NKIPyTensorRef):
        c = condition.backend_tensor
    elif np.isscalar(condition):
        c = as_graph_tensor(ctx, bool(condition), np.bool_)
    else:
        c = as_graph_tensor(ctx, np.asarray(condition).astype(bool), np.bool_)
    if np.dtype(c.dtype) != np.bool_:
        zero = as_graph_tensor(ctx, 0, c.dtype)
        if c.shape:
            zero = ctx.build_op("broadcast", [zero], c.shape, c.dtype, {"broadcast_dimensions": []})
        c = ctx.build_op("compare", [c, zero], c.shape, np.bool_, {"comparison_direction": "NE"})

    def operand(v):
        if isinstance(v, NKIPyTensorRef):
            return v.backend_tensor
        if np.isscalar(v):
            return as_graph_tensor(ctx, v, out_dt)
        return _const(ctx, v)

    a, b = operand(x), operand(y)
    shape = tuple(np.broadcast_shapes(tuple(c.shape), tuple(a.shape), tuple(b.shape)))
    if tuple(c.shape) != shape:
        c = broadcast_to_shape(ctx, c, shape)
    if tuple(a.shape) != shape:
        a = broadcast_to_shape(ctx, a, shape)
    if tuple(b.shape) != shape:
        b = broadcast_to_shape(ctx, b, shape)
    return NKIPyTensorRef(ctx.build_op("select", [c, a, b], shape, out_dt))


take = Op("take")


@take.impl("hlo")
def _take(x, indices, axis=None):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    if axis is None:
        t = ctx.build_op("reshape", [t], (int(np.prod(t.shape)),), t.dtype)
        axis = 0
    if axis < 0:
        axis += len(t.shape)
    if isinstance(indices, NKIPyTensorRef):
        it = indices.backend_tensor
    elif np.isscalar(indices):
        i = int(indices)
        if i < 0:
            i += t.shape[axis]
        it = as_graph_tensor(ctx, i, np.int32)
    elif isinstance(indices, (np.ndarray, list)):
        it = _const(ctx, np.asarray(indices), np.int32)
    else:
        raise ValueError("np.take only supports TensorRef, scalar, np.ndarray, or list as indices!")
    ishape = tuple(it.shape)
    out_shape = []
    for i, s in enumerate(t.shape):
        if i == axis:
            out_shape.extend(ishape)
        else:
            out_shape.append(s)
    out_shape = tuple(out_shape)
    offset_dims = [i for i in range(len(out_shape)) if i < axis or i >= axis + len(ishape)]
    sizes = list(t.shape)
    sizes[axis] = 1
    return NKIPyTensorRef(
        ctx.build_op(
            "gather",
            [t, it],
            out_shape,
            t.dtype,
            {
                "offset_dims": offset_dims,
                "collapsed_slice_dims": [axis],
                "start_index_map": [axis],
                "index_vector_dim": len(ishape),
                "slice_sizes": sizes,
                "indices_are_sorted": False,
            },
        )
    )


take_along_axis = Op("take_along_axis")


@take_along_axis.impl("hlo")
def _take_along_axis(x, indices, axis):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    if axis is None:
        t = ctx.build_op("reshape", [t], (int(np.prod(t.shape)),), t.dtype)
        axis = 0
    if axis < 0:
        axis += len(t.shape)
    if isinstance(indices, NKIPyTensorRef):
        it = indices.backend_tensor
    elif isinstance(indices, np.ndarray):
        it = _const(ctx, indices, np.int32)
    else:
        raise ValueError("take_along_axis only supports TensorRef or np.ndarray as indices!")
    rank = len(t.shape)
    if np.dtype(it.dtype) != np.int32:
        it = ctx.build_op("convert", [it], it.shape, np.int32)
    target = list(t.shape)
    target[axis] = it.shape[axis] if axis < len(it.shape) else 1
    target = tuple(target)
    if tuple(it.shape) != target:
        it = broadcast_to_shape(ctx, it, target)
    grids = []
    for d in range(rank):
        if d == axis:
            grids.append(it)
            continue
        g = _const(ctx, np.arange(t.shape[d], dtype=np.int32))
        gshape = [1] * rank
        gshape[d] = t.shape[d]
        g = ctx.build_op("reshape", [g], tuple(gshape), np.int32)
        grids.append(g)
    cols = []
    for g in grids:
        if tuple(g.shape) != target:
            g = broadcast_to_shape(ctx, g, target)
        cols.append(ctx.build_op("reshape", [g], target + (1,), np.int32))
    idx = ctx.build_op("concatenate", cols, target + (rank,), np.int32, {"dimension": rank})
    return NKIPyTensorRef(
        ctx.build_op(
            "gather",
            [t, idx],
            target,
            t.dtype,
            {
                "offset_dims": [],
                "collapsed_slice_dims": list(range(rank)),
                "start_index_map": list(range(rank)),
                "index_vector_dim": rank,
                "slice_sizes": [1] * rank,
                "indices_are_sorted": False,
            },
        )
    )


static_slice = Op("static_slice")


@static_slice.impl("hlo")
def _static_slice(x, start_indices, limit_indices, strides, squeeze_dims):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    shape = tuple((e - s + st - 1) // st for s, e, st in zip(start_indices, limit_indices, strides))
    r = ctx.build_op(
        "slice",
        [t],
        shape,
        t.dtype,
        {"start_indices": list(start_indices), "limit_indices": list(limit_indices), "strides": list(strides)},
    )
    if squeeze_dims:
        r = ctx.build_op("reshape", [r], tuple(s for i, s in enumerate(shape) if i not in squeeze_dims), t.dtype)
    return NKIPyTensorRef(r)


dynamic_update_slice = Op("dynamic_update_slice")


@dynamic_update_slice.impl("hlo")
def _dynamic_update_slice(x, value, start_indices, update_shape):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    update_shape = tuple(update_shape)
    if isinstance(value, NKIPyTensorRef):
        v = value.backend_tensor
    elif isinstance(value, (int, float)):
        v = ctx.build_op("constant", [], update_shape, t.dtype, {"value": np.full(update_shape, value, dtype=t.dtype)})
    elif isinstance(value, np.ndarray):
        v = ctx.build_op("constant", [], value.shape, value.dtype, {"value": value})
    else:
        v = value
    if tuple(v.shape) != update_shape:
        v = ctx.build_op("reshape", [v], update_shape, v.dtype)
    starts = [ctx.build_op("constant", [], (), np.int32, {"value": int(s)}) for s in start_indices]
    return NKIPyTensorRef(ctx.build_op("dynamic-update-slice", [t, v] + starts, t.shape, t.dtype, {}))


scatter_along_axis = Op("scatter_along_axis")


@scatter_along_axis.impl("hlo")
def _scatter_along_axis(x, indices, values, axis):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    base = ctx.build_op("copy", [t], t.shape, t.dtype)
    if axis < 0:
        axis += len(t.shape)
    if isinstance(indices, NKIPyTensorRef):
        it = indices.backend_tensor
    elif isinstance(indices, np.ndarray):
        it = _const(ctx, indices, np.int32)
    else:
        raise ValueError("scatter_along_axis requires TensorRef or np.ndarray indices")
    if isinstance(values, NKIPyTensorRef):
        vt = values.backend_tensor
    elif isinstance(values, np.ndarray):
        vt = _const(ctx, values, t.dtype)
    else:
        vt = as_graph_tensor(ctx, values, t.dtype)
    return NKIPyTensorRef(
        ctx.build_op(
            "scatter",
            [base, it, vt],
            base.shape,
            t.dtype,
            {
                "update_window_dims": [i for i in range(len(t.shape)) if i != axis],
                "inserted_window_dims": [axis],
                "scatter_dims_to_operand_dims": [axis],
                "index_vector_dim": len(it.shape),
                "update_computation": "assign",
                "indices_are_sorted": False,
                "unique_indices": False,
            },
        )
    )


put_along_axis = Op("put_along_axis")


@put_along_axis.impl("hlo")
def _put_along_axis(x, indices, values, axis):
    """Element scatter: arr[..., indices[i..], ...] = values[i..].

    Lowered, like the reference, to a scatter into the flattened array at
    offset = (fixed coordinates . strides) + index * stride[axis].
    """
    from nkipy_b200.core.ops.elementwise import add, multiply

    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    shape = tuple(t.shape)
    if axis is None:
        eff = (int(np.prod(shape)),)
        axis = 0
    else:
        if axis < 0:
            axis += len(shape)
        eff = shape
    if isinstance(indices, NKIPyTensorRef):
        it = indices.backend_tensor
    elif isinstance(indices, np.ndarray):
        it = _const(ctx, indices, np.int32)
    else:
        raise ValueError("put_along_axis only supports TensorRef or np.ndarray as indices!")
    if np.dtype(it.dtype) != np.int32:
        it = ctx.build_op("convert", [it], it.shape, np.int32)
    ishape = tuple(it.shape)
    if np.isscalar(values):
        vt = as_graph_tensor(ctx, values, t.dtype)
        if ishape:
            vt = ctx.build_op("broadcast", [vt], ishape, t.dtype, {"broadcast_dimensions": []})
    elif isinstance(values, NKIPyTensorRef):
        vt = values.backend_tensor
    elif isinstance(values, np.ndarray):
        vt = _const(ctx, values, t.dtype)
    else:
        raise ValueError("put_along_axis only supports scalar, TensorRef, or np.ndarray as values!")
    if tuple(vt.shape) != ishape:
        vt = ctx.build_op("reshape", [vt], ishape, vt.dtype)
    nd = len(eff)
    strides = [1] * nd
    for d in range(nd - 2, -1, -1):
        strides[d] = strides[d + 1] * eff[d + 1]
    fixed = np.zeros(ishape, dtype=np.int32)
    for d in range(nd):
        if d == axis:
            continue
        g = [1] * len(ishape)
        g[d] = ishape[d]
        fixed = fixed + np.arange(ishape[d], dtype=np.int32).reshape(g) * strides[d]
    flat_idx = add(NKIPyTensorRef(_const(ctx, fixed)), multiply(NKIPyTensorRef(it), int(strides[axis])))
    n = int(np.prod(ishape)) if ishape else 1
    fi = ctx.build_op("reshape", [flat_idx.backend_tensor], (n, 1), np.int32)
    fv = ctx.build_op("reshape", [vt], (n,), vt.dtype)
    total = int(np.prod(shape))
    base = ctx.build_op("copy", [t], shape, t.dtype)
    flat = ctx.build_op("reshape", [base], (total,), t.dtype)
    sc = ctx.build_op(
        "scatter",
        [flat, fi, fv],
        (total,),
        t.dtype,
        {
            "update_window_dims": [],
            "inserted_window_dims": [0],
            "scatter_dims_to_operand_dims": [0],
            "index_vector_dim": 1,
            "update_computation": "assign",
            "indices_are_sorted": False,
            "unique_indices": False,
        },
    )
    return NKIPyTensorRef(ctx.build_op("reshape", [sc], shape, t.dtype))


scatter_strided = Op("scatter_strided")


@scatter_strided.impl("hlo")
def _scatter_strided(x, value, scatter_indices_per_dim):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    vshape = tuple(len(i) for i in scatter_indices_per_dim)
    if isinstance(value, NKIPyTensorRef):
        v = value.backend_tensor
    elif isinstance(value, (int, float)):
        v = ctx.build_op("constant", [], vshape, t.dtype, {"value": np.full(vshape, value, dtype=t.dtype)})
    elif isinstance(value, np.ndarray):
        v = ctx.build_op("constant", [], value.shape, value.dtype, {"value": value})
    else:
        v = value
    pos = np.array(list(itertools.product(*scatter_indices_per_dim)), dtype=np.int32)
    it = ctx.build_op("constant", [], pos.shape, np.int32, {"value": pos})
    fv = ctx.build_op("reshape", [v], (pos.shape[0],), v.dtype)
    nd = len(t.shape)
    return NKIPyTensorRef(
        ctx.build_op(
            "scatter",
            [t, it, fv],
            t.shape,
            t.dtype,
            {
                "update_window_dims": [],
                "inserted_window_dims": list(range(nd)),
                "scatter_dims_to_operand_dims": list(range(nd)),
                "index_vector_dim": 1,
                "update_computation": "assign",
                "indices_are_sorted": False,
                "unique_indices": True,
            },
        )
    )
