"""Elementwise chains, broadcasts and reductions."""

import numpy as np

from nkipy_b200.core.specs import CommonTypes, KernelSpec, ShapeSpec, TensorInputSpec


def gelu_tanh(x):
    return 0.5 * x * (1.0 + np.tanh(0.7978845608 * (x + 0.044715 * x * x * x)))


def scaled_residual(x, y, z):
    return (x - y) * 0.5 + z[None, :]


def row_stats(x):
    m = np.mean(x, axis=-1, keepdims=True)
    v = np.mean(np.square(x - m), axis=-1, keepdims=True)
    return (x - m) / np.sqrt(v + 1e-5), np.max(x, axis=0)


def clip_where(x, lo):
    return np.where(x < lo, lo, np.minimum(x, 2.0)) * np.abs(x)


_F = CommonTypes.FLOATS
kernel_specs = [
    KernelSpec(gelu_tanh, [TensorInputSpec(dtype_spec=_F, shape_spec=ShapeSpec([(1, 512), (1, 2048)], (64, 1024)))],
               description="tanh GELU"),
    KernelSpec(scaled_residual, [TensorInputSpec(dtype_spec=_F, shape_spec=ShapeSpec([(1, 256), 96], (32, 96))),
                                 TensorInputSpec(dtype_spec=_F, shape_spec=ShapeSpec([(1, 256), 96], (32, 96))),
                                 TensorInputSpec(dtype_spec=_F, shape_spec=ShapeSpec([96], (96,)))],
               description="broadcast add of a row vector"),
    KernelSpec(row_stats, [TensorInputSpec(dtype_spec=CommonTypes.FLOATS,
                                           shape_spec=ShapeSpec([(1, 300), (2, 1024)], (48, 512)))],
               description="layer normalisation without weights, and a column maximum"),
    KernelSpec(clip_where, [TensorInputSpec(dtype_spec=_F, shape_spec=ShapeSpec([(1, 128), (1, 700)], (16, 700))),
                            TensorInputSpec(dtype_spec=_F, shape_spec=ShapeSpec([(1, 128), (1, 700)], (16, 700)))],
               description="select and clamp"),
]
