"""Collectives (reference: ``core/ops/collectives.py:14-233``).

Traced, each is one node (``all-gather``, ``all-reduce``, ``reduce-scatter``,
``all-to-all``) carrying ``replica_groups`` and the reduce op name; on the B200
runtime the node becomes an NCCL call on the plan's bound communicator.
The "cpu" implementations simulate ``world`` identical ranks, exactly as the
reference's CPU semantics do (``all_reduce(x) = x * world`` for add,
``all_gather`` tiles, ``reduce_scatter`` keeps rank 0's chunk).
"""

import numpy as np

from nkipy_b200.core.graph import get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef

_REDUCE_NAMES = {np.add: "add", np.multiply: "multiply", np.maximum: "maximum", np.minimum: "minimum"}


def _reduce_identical(data, world, reduce_op):
    if reduce_op is np.add:
        return data * world
    if reduce_op is np.multiply:
        return data**world
    return data.copy()


all_gather = Op("all_gather")


@all_gather.impl("cpu")
def _all_gather_cpu(data, all_gather_dim, replica_groups, **kwargs):
    world = len(replica_groups[0])
    return np.tile(data, tuple(world if i == all_gather_dim else 1 for i in range(data.ndim)))


@all_gather.impl("hlo")
def _all_gather(data, all_gather_dim, replica_groups, **kwargs):
    ctx = get_trace_context()
    shape = list(data.shape)
    if shape:
        shape[all_gather_dim] *= len(replica_groups[0])
    return NKIPyTensorRef(
        ctx.build_op(
            "all-gather",
            [data.backend_tensor],
            tuple(shape),
            data.dtype,
            {"all_gather_dim": all_gather_dim, "replica_groups": replica_groups},
        )
    )


all_reduce = Op("all_reduce")


@all_reduce.impl("cpu")
def _all_reduce_cpu(data, replica_groups, reduce_op=np.add, **kwargs):
    return _reduce_identical(data, len(replica_groups[0]), reduce_op)


@all_reduce.impl("hlo")
def _all_reduce(data, replica_groups, reduce_op=np.add, **kwargs):
    ctx = get_trace_context()
    return NKIPyTensorRef(
        ctx.build_op(
            "all-reduce",
            [data.backend_tensor],
            data.shape,
            data.dtype,
            {"replica_groups": replica_groups, "reduce_op": _REDUCE_NAMES.get(reduce_op, "add")},
        )
    )


reduce_scatter = Op("reduce_scatter")


@reduce_scatter.impl("cpu")
def _reduce_scatter_cpu(data, reduce_scatter_dim, replica_groups, reduce_op=np.add, **kwargs):
    world = len(replica_groups[0])
    reduced = _reduce_identical(data, world, reduce_op)
    return np.take(reduced, range(data.shape[reduce_scatter_dim] // world), axis=reduce_scatter_dim)


@reduce_scatter.impl("hlo")
def _reduce_scatter(data, reduce_scatter_dim, replica_groups, reduce_op=np.add, **kwargs):
    ctx = get_trace_context()
    shape = list(data.shape)
    if shape:
        shape[reduce_scatter_dim] //= len(replica_groups[0])
    return NKIPyTensorRef(
        ctx.build_op(
            "reduce-scatter",
            [data.backend_tensor],
            tuple(shape),
            data.dtype,
            {
                "reduce_scatter_dim": reduce_scatter_dim,
                "replica_groups": replica_groups,
                "reduce_op": _REDUCE_NAMES.get(reduce_op, "add"),
            },
        )
    )


all_to_all = Op("all_to_all")


@all_to_all.impl("cpu")
def _all_to_all_cpu(data, split_dimension, concat_dimension, replica_groups, **kwargs):
    chunks = np.split(data, len(replica_groups[0]), axis=split_dimension)
    return np.concatenate(chunks, axis=concat_dimension)


@all_to_all.impl("hlo")
def _all_to_all(data, split_dimension, concat_dimension, replica_groups, **kwargs):
    ctx = get_trace_context()
    return NKIPyTensorRef(
        ctx.build_op(
            "all-to-all",
            [data.backend_tensor],
            data.shape,
            data.dtype,
            {
                "split_dimension": split_dimension,
                "concat_dimension": concat_dimension,
                "replica_groups": replica_groups,
            },
        )
    )
