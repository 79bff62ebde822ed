"""NN-level ops (reference: ``core/ops/nn.py:12-160``).

``topk`` (last axis): a ``topk`` node plus two ``get-tuple-element`` nodes,
indices uint32; ascending order negates before and after, as the reference
does.  ``softmax`` and ``rms_norm`` are declared without an implementation in
the reference (kernels write them as NumPy compositions); here they trace to
the same compositions, which the planner fuses back into one kernel.
"""

import numpy as np

from nkipy_b200.core.graph import get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef

softmax = Op("softmax")


@softmax.impl("hlo")
def _softmax(x, axis=-1):
    from nkipy_b200.core.ops.elementwise import divide, exp, subtract
    from nkipy_b200.core.ops.reduce import max as _max
    from nkipy_b200.core.ops.reduce import sum as _sum

    e = exp(subtract(x, _max(x, axis=axis, keepdims=True)))
    return divide(e, _sum(e, axis=axis, keepdims=True))


rms_norm = Op("rms_norm")


@rms_norm.impl("hlo")
def _rms_norm(x, weight, eps=1e-6):
    from nkipy_b200.core.ops.elementwise import add, divide, multiply, sqrt
    from nkipy_b200.core.ops.reduce import mean

    ms = mean(multiply(x, x), axis=-1, keepdims=True)
    return multiply(divide(x, sqrt(add(ms, eps))), weight)


topk = Op("topk")


@topk.impl("cpu")
def _topk_cpu(x, k, axis=0, is_ascend=False, out=None, dtype=None):
    if axis < 0:
        axis += x.ndim
    key = x if is_ascend else -x
    idx = np.take(np.argpartition(key, k - 1, axis=axis), range(k), axis=axis)
    vals = np.take_along_axis(x, idx, axis=axis)
    order = np.argsort(vals if is_ascend else -vals, axis=axis)
    idx = np.take_along_axis(idx, order, axis=axis)
    vals = np.take_along_axis(vals, order, axis=axis)
    return vals, idx.astype(np.uint32)


@topk.impl("hlo")
def _topk(x, k, axis=0, is_ascend=False, out=None, dtype=None):
    if axis != -1 and axis != x.ndim - 1:
        raise NotImplementedError("the custom TopK op only supports last axis")
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    assert t.shape[-1] >= k, f"k={k} must be <= size of axis {len(t.shape) - 1} which is {t.shape[-1]}"
    shape = tuple(t.shape[:-1]) + (k,)
    src = ctx.build_op("negate", [t], t.shape, t.dtype) if is_ascend else t
    tup = ctx.build_op("topk", [src], shape, t.dtype, {"k": k, "largest": True, "is_tuple": True})
    vals = ctx.build_op("get-tuple-element", [tup], shape, t.dtype, {"tuple_index": 0})
    idx = ctx.build_op("get-tuple-element", [tup], shape, np.uint32, {"tuple_index": 1})
    if is_ascend:
        vals = ctx.build_op("negate", [vals], shape, t.dtype)
    return NKIPyTensorRef(vals), NKIPyTensorRef(idx)
