"""Convolutions (reference: ``core/ops/conv.py``): ``conv2d`` and ``conv3d``.

Layout as the reference: input (batch, in_channels, *spatial), weight
(out_channels, in_channels, *kernel), optional bias (out_channels,);
``stride``, ``padding`` (symmetric) and ``dilation`` are an int or one value
per spatial axis.

* "cpu": the direct-call semantics (``conv.py:133-228``): zero padding, then
  the correlation as one matrix product per batch over (channel, kernel
  offset) columns; dilation and groups other than 1 raise
  ``NotImplementedError`` as they do there.
* "hlo": one ``convolution`` node with the reference's attribute set
  (``conv.py:230-312``: window strides, symmetric padding pairs, rhs
  dilation, feature/batch group counts, NC-spatial dimension numbers) and
  output dtype = input dtype, then the bias as reshape + broadcast + add.
"""

import numpy as np

from nkipy_b200.core.graph import broadcast_to_shape, get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef


def _per_axis(value, n, name):
    if isinstance(value, (int, np.integer)):
        return (int(value),) * n
    if isinstance(value, (tuple, list)) and len(value) == n:
        return tuple(int(v) for v in value)
    raise ValueError(f"{name} must be an int or a tuple of {n} ints, got {value}")


def _out_extent(size, pad, kernel, stride, dil):
    return (size + 2 * pad - dil * (kernel - 1) - 1) // stride + 1


def _conv_cpu(n, x, w, bias, stride, padding, dilation, groups):
    stride = _per_axis(stride, n, "stride")
    padding = _per_axis(padding, n, "padding")
    dilation = _per_axis(dilation, n, "dilation")
    if dilation != (1,) * n:
        raise NotImplementedError(f"conv{n}d CPU backend does not support dilation != 1, got dilation={dilation}")
    if groups != 1:
        raise NotImplementedError(f"conv{n}d CPU backend does not support groups != 1, got groups={groups}")
    B, C = x.shape[:2]
    OC, kern = w.shape[0], tuple(w.shape[2:])
    xp = np.pad(x, ((0, 0), (0, 0)) + tuple((p, p) for p in padding)) if any(padding) else x
    # every kernel window of every channel: (B, C, *out, *kernel)
    win = np.lib.stride_tricks.sliding_window_view(xp, kern, axis=tuple(range(2, 2 + n)))
    win = win[(slice(None), slice(None)) + tuple(slice(None, None, s) for s in stride)]
    out_sp = win.shape[2:2 + n]
    # columns ordered (channel, kernel offsets), rows the output positions
    cols = np.moveaxis(win, tuple(range(2, 2 + n)), tuple(range(2 + n, 2 + 2 * n)))
    cols = cols.reshape(B, C * int(np.prod(kern)), int(np.prod(out_sp)))
    y = np.matmul(w.reshape(OC, -1), cols).reshape((B, OC) + tuple(out_sp))
    if bias is not None:
        y = y + bias.reshape((1, -1) + (1,) * n)
    return y


def _conv_hlo(n, x, w, bias, stride, padding, dilation, groups):
    ctx = get_trace_context()
    xt = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    wt = w.backend_tensor if isinstance(w, NKIPyTensorRef) else w
    stride = _per_axis(stride, n, "stride")
    padding = _per_axis(padding, n, "padding")
    dilation = _per_axis(dilation, n, "dilation")
    B, OC = xt.shape[0], wt.shape[0]
    spatial = tuple(
        _out_extent(xt.shape[2 + i], padding[i], wt.shape[2 + i], stride[i], dilation[i]) for i in range(n)
    )
    out_shape = (B, OC) + spatial
    sp = list(range(2, 2 + n))
    y = ctx.build_op(
        "convolution",
        [xt, wt],
        out_shape,
        xt.dtype,
        {
            "window_strides": list(stride),
            "padding": [(p, p) for p in padding],
            "lhs_dilation": [1] * n,
            "rhs_dilation": list(dilation),
            "feature_group_count": groups,
            "batch_group_count": 1,
            "input_batch_dimension": 0,
            "input_feature_dimension": 1,
            "input_spatial_dimensions": sp,
            "kernel_output_feature_dimension": 0,
            "kernel_input_feature_dimension": 1,
            "kernel_spatial_dimensions": sp,
            "output_batch_dimension": 0,
            "output_feature_dimension": 1,
            "output_spatial_dimensions": sp,
        },
    )
    if bias is not None:
        bt = bias.backend_tensor if isinstance(bias, NKIPyTensorRef) else bias
        br = ctx.build_op("reshape", [bt], (1, OC) + (1,) * n, bt.dtype)
        y = ctx.build_op("add", [y, broadcast_to_shape(ctx, br, out_shape)], out_shape, xt.dtype)
    return NKIPyTensorRef(y)


conv2d = Op("conv2d")


@conv2d.impl("cpu")
def _conv2d_cpu(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1, out=None, dtype=None):
    return _conv_cpu(2, input, weight, bias, stride, padding, dilation, groups)


@conv2d.impl("hlo")
def _conv2d_hlo(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1, out=None, dtype=None):
    return _conv_hlo(2, input, weight, bias, stride, padding, dilation, groups)


conv3d = Op("conv3d")


@conv3d.impl("cpu")
def _conv3d_cpu(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1, out=None, dtype=None):
    return _conv_cpu(3, input, weight, bias, stride, padding, dilation, groups)


@conv3d.impl("hlo")
def _conv3d_hlo(input, weight, bias=None, stride=1, padding=0, dilation=1, groups=1, out=None, dtype=None):
    return _conv_hlo(3, input, weight, bias, stride, padding, dilation, groups)
