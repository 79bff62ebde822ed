"""``NKIPyTensorRef``: the stand-in for an ndarray while a kernel is traced.

Behaviour follows the reference's ``nkipy/core/tensor.py``:

* Python operators map to the NumPy function of the same meaning
  (``tensor.py:51-200``), so ``a + b`` and ``np.add(a, b)`` trace alike;
* ``__array_ufunc__`` / ``__array_function__`` look the NumPy callable up in
  ``_tensor_apis`` and call the registered op (``tensor.py:420-456``); an
  unregistered function raises ``NotImplementedError``;
* ``__getitem__`` lowers static indices to ``slice`` (+ ``reshape`` for integer
  indices), a single tensor / list / array index to ``gather`` (after any static
  slice), and the ``a[np.arange(N), idx]`` form to ``take_along_axis``
  (``tensor.py:458-582``);
* ``__setitem__`` marks the reference mutated and rebinds it to the result of
  ``dynamic-update-slice`` / ``scatter`` (``tensor.py:627-851``); the tracer
  turns a mutated parameter into an aliased output.
"""

from __future__ import annotations

import inspect
import math
from typing import Tuple

import numpy as np

_INTERNAL_DIR = "nkipy_b200/"


def find_source_loc():
    """First stack frame outside this package: the user line being traced."""
    try:
        frame = inspect.currentframe().f_back.f_back
        while frame is not None and _INTERNAL_DIR in frame.f_code.co_filename:
            frame = frame.f_back
        if frame is None:
            return None
        return (frame.f_code.co_filename, frame.f_lineno)
    except Exception:  # pragma: no cover - best effort only
        return None


def _set_loc(loc):
    from nkipy_b200.core.backend import set_source_location

    set_source_location(loc)


def _ops():
    from nkipy_b200.core import ops

    return ops


class TensorArithmeticMixin:
    def __add__(self, o):
        return np.add(self, o)

    def __sub__(self, o):
        return np.subtract(self, o)

    def __mul__(self, o):
        return np.multiply(self, o)

    def __truediv__(self, o):
        return np.divide(self, o)

    def __floordiv__(self, o):
        return np.floor_divide(self, o)

    def __mod__(self, o):
        return np.mod(self, o)

    def __pow__(self, o):
        return np.power(self, o)

    def __matmul__(self, o):
        return np.matmul(self, o)

    def __radd__(self, o):
        return np.add(o, self)

    def __rsub__(self, o):
        return np.subtract(o, self)

    def __rmul__(self, o):
        return np.multiply(o, self)

    def __rtruediv__(self, o):
        return np.divide(o, self)

    def __rfloordiv__(self, o):
        return np.floor_divide(o, self)

    def __rmod__(self, o):
        return np.mod(o, self)

    def __rpow__(self, o):
        return np.power(o, self)

    def __rmatmul__(self, o):
        return np.matmul(o, self)

    def __abs__(self):
        return np.abs(self)

    def __neg__(self):
        return np.negative(self)

    def __pos__(self):
        return np.copy(self)

    # in-place operators produce a new node, like the reference
    __iadd__ = __add__
    __isub__ = __sub__
    __imul__ = __mul__
    __itruediv__ = __truediv__
    __ifloordiv__ = __floordiv__
    __imod__ = __mod__
    __ipow__ = __pow__
    __imatmul__ = __matmul__

    def __lt__(self, o):
        return np.less(self, o)

    def __le__(self, o):
        return np.less_equal(self, o)

    def __gt__(self, o):
        return np.greater(self, o)

    def __ge__(self, o):
        return np.greater_equal(self, o)

    def __eq__(self, o):
        return np.equal(self, o)

    def __ne__(self, o):
        return np.not_equal(self, o)

    def __and__(self, o):
        return np.bitwise_and(self, o)

    def __or__(self, o):
        return np.bitwise_or(self, o)

    def __xor__(self, o):
        return np.bitwise_xor(self, o)

    def __invert__(self):
        return np.invert(self)

    def __rand__(self, o):
        return np.bitwise_and(o, self)

    def __ror__(self, o):
        return np.bitwise_or(o, self)

    def __rxor__(self, o):
        return np.bitwise_xor(o, self)

    __hash__ = object.__hash__


class TensorOperationMixin:
    def transpose(self, *axes):
        if not axes:
            return np.transpose(self, axes=None)
        if len(axes) == 1 and isinstance(axes[0], (tuple, list)):
            return np.transpose(self, axes[0])
        return np.transpose(self, axes)

    def reshape(self, *shape):
        if not shape:
            raise TypeError("reshape() takes at least 1 argument (0 given)")
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            return np.reshape(self, shape[0])
        return np.reshape(self, shape)

    def mean(self, axis=None, keepdims=False, **kw):
        return np.mean(self, axis=axis, keepdims=keepdims, **kw)

    def sum(self, axis=None, keepdims=False, **kw):
        return np.sum(self, axis=axis, keepdims=keepdims, **kw)

    def var(self, axis=None, keepdims=False, **kw):
        return np.var(self, axis=axis, keepdims=keepdims, **kw)

    def std(self, axis=None, keepdims=False, **kw):
        return np.std(self, axis=axis, keepdims=keepdims, **kw)

    def squeeze(self, axis=None):
        return np.squeeze(self, axis=axis)

    def max(self, axis=None, keepdims=False, **kw):
        return np.max(self, axis=axis, keepdims=keepdims, **kw)

    def min(self, axis=None, keepdims=False, **kw):
        return np.min(self, axis=axis, keepdims=keepdims, **kw)

    def copy(self):
        return np.copy(self)

    def clip(self, a_min=None, a_max=None):
        return np.clip(self, a_min, a_max)

    def ravel(self):
        return np.reshape(self, (-1,))

    def swapaxes(self, a1, a2):
        return np.swapaxes(self, a1, a2)

    def prod(self, axis=None, keepdims=False, **kw):
        return np.prod(self, axis=axis, keepdims=keepdims, **kw)

    def argmin(self, axis=None, **kw):
        return np.argmin(self, axis=axis, **kw)

    def argmax(self, axis=None, **kw):
        return np.argmax(self, axis=axis, **kw)


def _expand_ellipsis(indices: tuple, ndim: int) -> tuple:
    n_ell = sum(1 for i in indices if i is Ellipsis)
    if n_ell == 0:
        return indices
    if n_ell > 1:
        raise IndexError("an index can only have a single ellipsis (...)")
    n_real = sum(1 for i in indices if i is not None and i is not Ellipsis)
    fill = ndim - n_real
    if fill < 0:
        raise IndexError(
            f"too many indices for tensor: tensor is {ndim}-dimensional, but {n_real} were given"
        )
    out = ()
    for i in indices:
        out += (slice(None),) * fill if i is Ellipsis else (i,)
    return out


def _strip_newaxis(indices: tuple):
    kept, new_axes, pos = [], [], 0
    for i in indices:
        if i is None:
            new_axes.append(pos)
            pos += 1
        elif isinstance(i, (int, np.integer)):
            kept.append(int(i))
        else:
            kept.append(i)
            pos += 1
    return tuple(kept), new_axes


def _norm_slice(idx: slice, size: int):
    start = 0 if idx.start is None else int(idx.start)
    stop = size if idx.stop is None else int(idx.stop)
    step = 1 if idx.step is None else int(idx.step)
    if start < 0:
        start += size
    if stop < 0:
        stop += size
    return start, stop, step


class NKIPyTensorRef(TensorArithmeticMixin, TensorOperationMixin):
    """Reference to a traced graph tensor, usable where NumPy expects an array."""

    __slots__ = ("backend_tensor", "_shape", "_dtype", "_name", "_original_parameter", "_is_mutated")
    _tensor_apis = {}

    def __init__(self, backend_tensor, name: str = None):
        self.backend_tensor = backend_tensor
        self._shape = tuple(backend_tensor.shape)
        self._dtype = np.dtype(backend_tensor.dtype)
        self._name = name
        self._original_parameter = None
        self._is_mutated = False

    @property
    def name(self):
        return self._name

    @property
    def shape(self) -> Tuple[int, ...]:
        return self._shape

    @property
    def dtype(self):
        return self._dtype

    @property
    def ndim(self) -> int:
        return len(self._shape)

    @property
    def T(self):
        return self.transpose()

    @property
    def size(self) -> int:
        return math.prod(self._shape)

    @property
    def strides(self):
        out, step = [], self._dtype.itemsize
        for s in reversed(self._shape):
            out.append(step)
            step *= s
        return tuple(reversed(out))

    def __len__(self):
        if not self._shape:
            raise TypeError("len() of unsized object")
        return self._shape[0]

    def __array__(self, dtype=None, copy=None):
        raise TypeError(
            "NKIPyTensorRef cannot be converted to a numpy array: it only exists as a node "
            "of the traced graph."
        )

    def __repr__(self):
        return f"NKIPyTensorRef(name={self._name}, shape={self.shape}, dtype={self.dtype})"

    def _rebind(self, result):
        self.backend_tensor = result.backend_tensor
        self._shape = tuple(result.shape)
        self._dtype = np.dtype(result.dtype)

    def astype(self, dtype):
        _set_loc(find_source_loc())
        try:
            return _ops().astype(self, dtype)
        finally:
            _set_loc(None)

    def __array_ufunc__(self, ufunc, method, *inputs, **kwargs):
        if method != "__call__":
            return NotImplemented
        _set_loc(find_source_loc())
        try:
            return self.__array_function__(ufunc, (), inputs, kwargs)
        finally:
            _set_loc(None)

    def __array_function__(self, func, types, args, kwargs):
        impl = self._tensor_apis.get(func)
        if impl is None:
            raise NotImplementedError(
                f"NumPy function '{getattr(func, '__name__', func)}' has not been implemented in NKIPy."
            )
        _set_loc(find_source_loc())
        try:
            return impl(*args, **kwargs)
        finally:
            _set_loc(None)

    # -- indexing ---------------------------------------------------------
    def __getitem__(self, indices):
        ops = _ops()
        _set_loc(find_source_loc())
        try:
            if not isinstance(indices, tuple):
                indices = (indices,)
            indices = _expand_ellipsis(indices, self.ndim)
            indices, new_axes = _strip_newaxis(indices)
            indices = indices + (slice(None),) * (self.ndim - len(indices))
            dyn_types = (NKIPyTensorRef, np.ndarray, list)
            for idx in indices:
                if isinstance(idx, (NKIPyTensorRef, np.ndarray)) and np.dtype(idx.dtype) == np.bool_:
                    raise NotImplementedError(
                        "Boolean indexing is not supported: a boolean mask gives a data-dependent shape."
                    )
            dyn = [(d, i) for d, i in enumerate(indices) if isinstance(i, dyn_types)]
            if dyn:
                result = None
                if len(dyn) == 2:
                    result = self._diagonal_gather(dyn, ops)
                if result is None:
                    if len(dyn) > 1:
                        raise ValueError("Only one tensor index is currently supported")
                    dim, value = dyn[0]
                    static = tuple(slice(None) if d == dim else i for d, i in enumerate(indices))
                    needs_static = any(
                        not (isinstance(i, slice) and i == slice(None)) for d, i in enumerate(static) if d != dim
                    )
                    if needs_static:
                        base = self._static_slice(static)
                        dropped = sum(1 for i in static[:dim] if isinstance(i, int))
                        result = ops.take(base, value, axis=dim - dropped)
                    else:
                        result = ops.take(self, value, axis=dim)
            else:
                result = self._static_slice(indices)
            if new_axes:
                result = ops.expand_dims(result, axis=new_axes)
            return result
        finally:
            _set_loc(None)

    def _diagonal_gather(self, dyn, ops):
        (d1, i1), (d2, i2) = dyn

        def is_arange(idx, n):
            return (
                isinstance(idx, np.ndarray)
                and idx.ndim == 1
                and len(idx) == n
                and np.array_equal(idx, np.arange(n))
            )

        if is_arange(i1, self.shape[d1]):
            ar_dim, g_dim, idx = d1, d2, i2
        elif is_arange(i2, self.shape[d2]):
            ar_dim, g_dim, idx = d2, d1, i1
        else:
            return None
        shp = [1] * self.ndim
        shp[ar_dim] = self.shape[ar_dim]
        if isinstance(idx, NKIPyTensorRef):
            idx = ops.reshape(idx, tuple(shp))
        else:
            idx = np.asarray(idx).reshape(shp)
        return ops.squeeze(ops.take_along_axis(self, idx, axis=g_dim), axis=g_dim)

    def _static_slice(self, indices):
        starts, limits, steps, squeeze = [], [], [], []
        for d, idx in enumerate(indices):
            if isinstance(idx, slice):
                s, e, st = _norm_slice(idx, self.shape[d])
                starts.append(s)
                limits.append(e)
                steps.append(st)
            elif isinstance(idx, int):
                i = idx + self.shape[d] if idx < 0 else idx
                starts.append(i)
                limits.append(i + 1)
                steps.append(1)
                squeeze.append(d)
            else:
                raise ValueError(f"Unsupported index type in static slicing: {type(idx)}")
        return _ops().static_slice(self, starts, limits, steps, squeeze)

    def __setitem__(self, indices, value):
        ops = _ops()
        _set_loc(find_source_loc())
        try:
            if not isinstance(indices, tuple):
                indices = (indices,)
            if any(i is None for i in indices):
                raise IndexError(
                    "cannot use a newaxis (None) in a setitem expression. Use np.expand_dims() on the value instead."
                )
            indices = _expand_ellipsis(indices, self.ndim)
            indices = indices + (slice(None),) * (self.ndim - len(indices))
            indices = tuple(int(i) if isinstance(i, np.integer) else i for i in indices)
            self._is_mutated = True
            tensor_dims = [d for d, i in enumerate(indices) if isinstance(i, NKIPyTensorRef)]
            if tensor_dims:
                if len(tensor_dims) > 1:
                    raise ValueError("Only one tensor index is currently supported")
                d = tensor_dims[0]
                result = ops.scatter_along_axis(self, indices[d], value, axis=d)
                if result is not None:
                    self._rebind(result)
                return
            strided = any(isinstance(i, slice) and i.step not in (None, 1) for i in indices)
            if strided:
                per_dim = []
                for d, idx in enumerate(indices):
                    if isinstance(idx, slice):
                        s, e, st = _norm_slice(idx, self.shape[d])
                        per_dim.append(list(range(s, e, st)))
                    else:
                        per_dim.append([idx + self.shape[d] if idx < 0 else idx])
                self._rebind(ops.scatter_strided(self, value, per_dim))
                return
            upd_shape, starts = [], []
            for d, idx in enumerate(indices):
                if isinstance(idx, slice):
                    s, e, st = _norm_slice(idx, self.shape[d])
                    upd_shape.append((e - s + st - 1) // st)
                    starts.append(s)
                else:
                    i = idx + self.shape[d] if idx < 0 else idx
                    upd_shape.append(1)
                    starts.append(i)
            self._rebind(ops.dynamic_update_slice(self, value, starts, tuple(upd_shape)))
        finally:
            _set_loc(None)
