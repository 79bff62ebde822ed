"""Index selection, argmax and in-place row updates."""

import numpy as np

from nkipy_b200.core.specs import CommonTypes, KernelSpec, ShapeSpec, TensorInputSpec, TypeSpec

_I32 = TypeSpec(allowed=[np.int32], default=np.int32)


def embedding_lookup(table, ids):
    return np.take(table, ids, axis=0) * np.float32(np.sqrt(table.shape[1]))


def gather_rows_by_argmax(x, table):
    best = np.argmax(x, axis=-1)
    return np.take(table, best, axis=0), best


def take_along_last(x, idx):
    return np.take_along_axis(x, idx, axis=-1)


def update_row(cache, row, pos):
    cache[pos] = row
    return cache * 2.0


kernel_specs = [
    KernelSpec(embedding_lookup, [
        TensorInputSpec(dtype_spec=CommonTypes.FLOATS, shape_spec=ShapeSpec([(1000, 4096), (16, 512)], (1000, 256))),
        TensorInputSpec(dtype_spec=_I32, shape_spec=ShapeSpec([(1, 64)], (37,)),
                        default_value=np.array([3, 0, 999, 17, 17, 500] * 6 + [1], np.int32)),
    ], description="token embedding lookup"),
    KernelSpec(gather_rows_by_argmax, [
        TensorInputSpec(dtype_spec=CommonTypes.FLOATS, shape_spec=ShapeSpec([(1, 64), 50], (20, 50))),
        TensorInputSpec(dtype_spec=CommonTypes.FLOATS, shape_spec=ShapeSpec([50, (1, 256)], (50, 64))),
    ], description="argmax, then a row gather"),
    KernelSpec(take_along_last, [
        TensorInputSpec(dtype_spec=CommonTypes.FLOATS, shape_spec=ShapeSpec([12, 40], (12, 40))),
        TensorInputSpec(dtype_spec=_I32, shape_spec=ShapeSpec([12, 5], (12, 5)),
                        default_value=(np.arange(60, dtype=np.int32).reshape(12, 5) * 7) % 40),
    ], description="take_along_axis on the last axis"),
    KernelSpec(update_row, [
        TensorInputSpec(dtype_spec=CommonTypes.FLOATS, shape_spec=ShapeSpec([16, 64], (16, 64))),
        TensorInputSpec(dtype_spec=CommonTypes.FLOATS, shape_spec=ShapeSpec([64], (64,))),
        TensorInputSpec(dtype_spec=_I32, shape_spec=ShapeSpec([1], (1,)), default_value=np.array([5], np.int32)),
    ], description="row written in place at a run-time position"),
]


def argmax_int(x):
    return np.argmax(x, axis=-1)


kernel_specs.append(KernelSpec(argmax_int, [
    TensorInputSpec(dtype_spec=CommonTypes.INTS, shape_spec=ShapeSpec([(1, 40), (1, 300)], (17, 300)))],
    description="argmax of integers (first occurrence)"))
