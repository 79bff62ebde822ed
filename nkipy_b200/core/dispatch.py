"""NumPy callable -> op table used by ``NKIPyTensorRef.__array_function__``.

Same coverage as the reference's ``core/_numpy_dispatch.py:27-159``: anything
not listed (``np.einsum``, ``np.arctan2``, ``np.positive`` ...) raises
``NotImplementedError`` while tracing.
"""

import numpy as np

from nkipy_b200.core.tensor import NKIPyTensorRef

_registered = False


def _table(ops):
    return {
        np.add: ops.add,
        np.subtract: ops.subtract,
        np.multiply: ops.multiply,
        np.divide: ops.divide,
        np.power: ops.power,
        np.maximum: ops.maximum,
        np.minimum: ops.minimum,
        np.bitwise_and: ops.bitwise_and,
        np.bitwise_or: ops.bitwise_or,
        np.bitwise_xor: ops.bitwise_xor,
        np.logaddexp: ops.logaddexp,
        np.remainder: ops.remainder,
        np.mod: ops.remainder,
        np.floor_divide: ops.floor_divide,
        np.equal: ops.equal,
        np.not_equal: ops.not_equal,
        np.greater: ops.greater,
        np.greater_equal: ops.greater_equal,
        np.less: ops.less,
        np.less_equal: ops.less_equal,
        np.logical_and: ops.logical_and,
        np.logical_or: ops.logical_or,
        np.logical_xor: ops.logical_xor,
        np.abs: ops.abs,
        np.exp: ops.exp,
        np.log: ops.log,
        np.sqrt: ops.sqrt,
        np.square: ops.square,
        np.negative: ops.negative,
        np.reciprocal: ops.reciprocal,
        np.sin: ops.sin,
        np.cos: ops.cos,
        np.tan: ops.tan,
        np.arctan: ops.arctan,
        np.tanh: ops.tanh,
        np.ceil: ops.ceil,
        np.floor: ops.floor,
        np.rint: ops.rint,
        np.trunc: ops.trunc,
        np.sign: ops.sign,
        np.invert: ops.invert,
        np.bitwise_not: ops.bitwise_not,
        np.logical_not: ops.logical_not,
        np.clip: ops.clip,
        np.log1p: ops.log1p,
        np.log2: ops.log2,
        np.expm1: ops.expm1,
        np.round: ops.round_,
        np.around: ops.round_,
        np.isnan: ops.isnan,
        np.isfinite: ops.isfinite,
        np.sum: ops.sum,
        np.max: ops.max,
        np.min: ops.min,
        np.mean: ops.mean,
        np.any: ops.any,
        np.var: ops.var,
        np.std: ops.std,
        np.argmax: ops.argmax,
        np.argmin: ops.argmin,
        np.cumsum: ops.cumsum,
        np.prod: ops.prod,
        np.count_nonzero: ops.count_nonzero,
        np.matmul: ops.matmul,
        np.dot: ops.dot,
        np.linalg.norm: ops.norm,
        np.outer: ops.outer,
        np.trace: ops.trace,
        np.reshape: ops.reshape,
        np.transpose: ops.transpose,
        np.expand_dims: ops.expand_dims,
        np.concatenate: ops.concatenate,
        np.split: ops.split,
        np.copy: ops.copy,
        np.repeat: ops.repeat,
        np.squeeze: ops.squeeze,
        np.pad: ops.pad,
        np.swapaxes: ops.swapaxes,
        np.stack: ops.stack,
        np.diff: ops.diff,
        np.flip: ops.flip,
        np.tile: ops.tile,
        np.roll: ops.roll,
        np.tril: ops.tril,
        np.triu: ops.triu,
        np.diag: ops.diag,
        np.zeros_like: ops.zeros_like,
        np.ones_like: ops.ones_like,
        np.empty_like: ops.empty_like,
        np.full_like: ops.full_like,
        np.where: ops.where,
        np.take: ops.take,
        np.take_along_axis: ops.take_along_axis,
        np.broadcast_to: ops.broadcast_to,
        np.copyto: ops.copyto,
    }


def register_all_numpy_apis():
    global _registered
    if _registered:
        return
    from nkipy_b200.core import ops

    for np_fn, op in _table(ops).items():
        NKIPyTensorRef._tensor_apis[np_fn] = op

    def _put_along_axis_inplace(arr, indices, values, axis):
        # np.put_along_axis mutates its argument and returns None: rebind the
        # reference so the tracer sees the mutation (reference
        # _numpy_dispatch.py:143-154).
        res = ops.put_along_axis(arr, indices, values, axis)
        if isinstance(arr, NKIPyTensorRef) and res is not None:
            arr._rebind(res)
            arr._is_mutated = True

    NKIPyTensorRef._tensor_apis[np.put_along_axis] = _put_along_axis_inplace
    _registered = True
