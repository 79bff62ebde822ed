"""Layout ops (reference: ``core/ops/transform.py:14-876``).

``reshape``/``expand_dims``/``squeeze`` are ``reshape`` nodes (free on the
device: every buffer is dense row-major), ``transpose`` carries a
``permutation``, ``split`` emits ``slice`` nodes, ``concatenate`` one node with
``dimension``, ``repeat`` is ``broadcast`` + ``reshape``, ``astype`` is
``convert`` (or ``copy`` when the dtype is unchanged), ``pad`` is ``pad`` with
a ``padding_config`` (``edge`` mode: slices + concatenates), ``flip`` is a
``take`` with reversed indices, ``tile`` is reshape/broadcast/reshape and
``roll`` two slices and a concatenate.
"""

import numpy as np

from nkipy_b200.core.graph import as_graph_tensor, broadcast_to_shape, get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef


def _bt(x):
    return x.backend_tensor if isinstance(x, NKIPyTensorRef) else x


reshape = Op("reshape")


@reshape.impl("hlo")
def _reshape(x, newshape):
    ctx = get_trace_context()
    t = _bt(x)
    if isinstance(newshape, (int, np.integer)):
        newshape = (int(newshape),)
    newshape = tuple(int(d) for d in newshape)
    total = int(np.prod(t.shape))
    if -1 in newshape:
        known = int(np.prod([d for d in newshape if d != -1]))
        assert known > 0, "Cannot reshape to a size of 0"
        assert total % known == 0, f"Cannot reshape array of size {total} into shape {newshape}"
        newshape = tuple(total // known if d == -1 else d for d in newshape)
    if int(np.prod(newshape)) != total:
        raise ValueError(f"Cannot reshape array of size {total} into shape {newshape}")
    return NKIPyTensorRef(ctx.build_op("reshape", [t], newshape, t.dtype))


transpose = Op("transpose")


@transpose.impl("hlo")
def _transpose(x, axes=None, out=None, dtype=None):
    ctx = get_trace_context()
    t = _bt(x)
    if axes is None:
        axes = list(range(len(t.shape)))[::-1]
    axes = [int(a) + len(t.shape) if int(a) < 0 else int(a) for a in axes]
    shape = tuple(t.shape[a] for a in axes)
    return NKIPyTensorRef(ctx.build_op("transpose", [t], shape, t.dtype, {"permutation": axes}))


swapaxes = Op("swapaxes")


@swapaxes.impl("hlo")
def _swapaxes(x, axis1, axis2):
    nd = len(x.shape)
    a1 = axis1 + nd if axis1 < 0 else axis1
    a2 = axis2 + nd if axis2 < 0 else axis2
    if not (0 <= a1 < nd and 0 <= a2 < nd):
        raise np.exceptions.AxisError(f"axis is out of bounds for array of dimension {nd}")
    perm = list(range(nd))
    perm[a1], perm[a2] = perm[a2], perm[a1]
    return transpose(x, axes=perm)


expand_dims = Op("expand_dims")


@expand_dims.impl("hlo")
def _expand_dims(x, axis):
    ctx = get_trace_context()
    t = _bt(x)
    rank = len(t.shape)
    shape = list(t.shape)
    if isinstance(axis, (list, tuple)):
        final = rank + len(axis)
        axes = []
        for a in axis:
            a = a + final if a < 0 else a
            if a < 0 or a > final - 1:
                raise ValueError(f"axis {a} is out of bounds for array of dimension {final}")
            axes.append(a)
        if len(set(axes)) != len(axes):
            raise ValueError("repeated axis in expand_dims")
        for a in sorted(axes):
            shape.insert(a, 1)
    else:
        a = axis + rank + 1 if axis < 0 else axis
        if a < 0 or a > rank:
            raise ValueError(f"axis {a} is out of bounds for array of dimension {rank}")
        shape.insert(a, 1)
    return NKIPyTensorRef(ctx.build_op("reshape", [t], tuple(shape), t.dtype))


concatenate = Op("concatenate")


@concatenate.impl("hlo")
def _concatenate(tensors, axis=0):
    from nkipy_b200.core.ops.creation import constant

    ctx = get_trace_context()
    ts = []
    for t in tensors:
        if isinstance(t, NKIPyTensorRef):
            ts.append(t.backend_tensor)
        elif isinstance(t, np.ndarray):
            ts.append(constant(t).backend_tensor)
        else:
            ts.append(t)
    if not ts:
        raise ValueError("Need at least one tensor to concatenate")
    if len(ts) == 1:
        return NKIPyTensorRef(ctx.build_op("copy", [ts[0]], ts[0].shape, ts[0].dtype))
    nd = len(ts[0].shape)
    ax = axis + nd if axis < 0 else axis
    if ax < 0 or ax >= nd:
        raise ValueError(f"axis {ax} is out of bounds for array of dimension {nd}")
    shape = list(ts[0].shape)
    shape[ax] = sum(t.shape[ax] for t in ts)
    dt = np.dtype(ts[0].dtype)
    for t in ts[1:]:
        dt = np.result_type(dt, t.dtype)
    return NKIPyTensorRef(ctx.build_op("concatenate", ts, tuple(shape), dt, {"dimension": ax}))


stack = Op("stack")


@stack.impl("hlo")
def _stack(arrays, axis=0, out=None, dtype=None):
    return concatenate([expand_dims(a, axis=axis) for a in arrays], axis=axis)


def _slice_node(ctx, t, starts, limits, strides=None):
    nd = len(t.shape)
    strides = strides or [1] * nd
    shape = tuple((e - s + st - 1) // st for s, e, st in zip(starts, limits, strides))
    return ctx.build_op(
        "slice", [t], shape, t.dtype, {"start_indices": list(starts), "limit_indices": list(limits), "strides": list(strides)}
    )


split = Op("split")


@split.impl("hlo")
def _split(x, indices_or_sections, axis=0):
    ctx = get_trace_context()
    t = _bt(x)
    nd = len(t.shape)
    ax = axis + nd if axis < 0 else axis
    if ax < 0 or ax >= nd:
        raise ValueError(f"axis {ax} is out of bounds for array of dimension {nd}")
    size = t.shape[ax]
    if isinstance(indices_or_sections, (int, np.integer)):
        n = int(indices_or_sections)
        if n <= 0:
            raise ValueError("Number of sections must be larger than 0")
        if size % n:
            raise ValueError("Array split does not result in an equal division")
        cuts = [i * (size // n) for i in range(1, n)]
    else:
        cuts = [int(c) for c in indices_or_sections]
    bounds = [0] + cuts + [size]
    out = []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        starts = [0] * nd
        limits = list(t.shape)
        starts[ax], limits[ax] = lo, hi
        out.append(NKIPyTensorRef(_slice_node(ctx, t, starts, limits)))
    return out


copy = Op("copy")


@copy.impl("hlo")
def _copy(x, out=None, dtype=None):
    ctx = get_trace_context()
    t = _bt(x)
    return NKIPyTensorRef(ctx.build_op("copy", [t], t.shape, t.dtype))


repeat = Op("repeat")


@repeat.impl("hlo")
def _repeat(x, repeats, axis=None):
    ctx = get_trace_context()
    t = _bt(x)
    if axis is None:
        t = ctx.build_op("reshape", [t], (int(np.prod(t.shape)),), t.dtype)
        axis = 0
    if axis < 0:
        axis += len(t.shape)
    if not isinstance(repeats, (int, np.integer)):
        raise TypeError(
            f"Only compile-time-known integer repeats are supported, got {type(repeats).__name__}."
        )
    repeats = int(repeats)
    final = list(t.shape)
    final[axis] *= repeats
    bshape = list(t.shape)
    bshape.insert(axis + 1, repeats)
    bdims = [i if i <= axis else i + 1 for i in range(len(t.shape))]
    b = ctx.build_op("broadcast", [t], tuple(bshape), t.dtype, {"broadcast_dimensions": bdims})
    return NKIPyTensorRef(ctx.build_op("reshape", [b], tuple(final), t.dtype))


broadcast_to = Op("broadcast_to")


@broadcast_to.impl("hlo")
def _broadcast_to(x, shape, out=None, dtype=None):
    ctx = get_trace_context()
    t = _bt(x)
    target = (int(shape),) if isinstance(shape, (int, np.integer)) else tuple(int(s) for s in shape)
    if tuple(t.shape) == target:
        return NKIPyTensorRef(ctx.build_op("copy", [t], t.shape, t.dtype))
    return NKIPyTensorRef(broadcast_to_shape(ctx, t, target))


copyto = Op("copyto")


squeeze = Op("squeeze")


@squeeze.impl("hlo")
def _squeeze(x, axis=None):
    shape = tuple(x.shape)
    nd = len(shape)
    if axis is None:
        new = tuple(s for s in shape if s != 1)
    else:
        axes = (axis,) if isinstance(axis, int) else tuple(axis)
        axes = tuple(a + nd if a < 0 else a for a in axes)
        for a in axes:
            if shape[a] != 1:
                raise ValueError(
                    f"cannot select an axis to squeeze out which has size not equal to one, got shape[{a}] = {shape[a]}"
                )
        new = tuple(s for i, s in enumerate(shape) if i not in axes)
    if new == shape:
        return x
    return reshape(x, new)


astype = Op("astype")


@astype.impl("hlo")
def _astype(x, dtype):
    ctx = get_trace_context()
    t = _bt(x)
    dtype = np.dtype(dtype)
    if np.dtype(t.dtype) == dtype:
        return NKIPyTensorRef(ctx.build_op("copy", [t], t.shape, t.dtype))
    return NKIPyTensorRef(ctx.build_op("convert", [t], t.shape, dtype))


def _single_index_slice(x, dim, index):
    ctx = get_trace_context()
    t = _bt(x)
    nd = len(t.shape)
    starts = [0] * nd
    limits = list(t.shape)
    starts[dim], limits[dim] = index, index + 1
    s = _slice_node(ctx, t, starts, limits)
    return NKIPyTensorRef(ctx.build_op("reshape", [s], tuple(v for i, v in enumerate(t.shape) if i != dim), t.dtype))


pad = Op("pad")


@pad.impl("hlo")
def _pad(x, pad_width, mode="constant", constant_values=0, **kwargs):
    ctx = get_trace_context()
    t = _bt(x)
    nd = len(t.shape)
    pw = np.asarray(pad_width)
    if pw.ndim == 0:
        pw = np.broadcast_to(pw, (nd, 2))
    elif pw.ndim == 1:
        if len(pw) == 2:
            pw = np.broadcast_to(pw, (nd, 2))
        else:
            pw = np.array([[p, p] for p in pw])
            if len(pw) != nd:
                raise ValueError(f"pad_width must have length {nd} to match array dimensions, got {len(pw)}")
    if pw.ndim == 2 and len(pw) == 1:
        pw = np.broadcast_to(pw, (nd, 2))
    pw = [(int(pw[i, 0]), int(pw[i, 1])) for i in range(nd)]
    if mode == "constant":
        cfg = [(lo, hi, 0) for lo, hi in pw]
        shape = tuple(s + lo + hi for s, (lo, hi) in zip(t.shape, pw))
        val = as_graph_tensor(ctx, constant_values, t.dtype)
        return NKIPyTensorRef(ctx.build_op("pad", [t, val], shape, t.dtype, {"padding_config": cfg}))
    if mode == "edge":
        res = x if isinstance(x, NKIPyTensorRef) else NKIPyTensorRef(t)
        for d in range(nd):
            lo, hi = pw[d]
            if lo == 0 and hi == 0:
                continue
            parts = []
            if lo > 0:
                parts.append(repeat(expand_dims(_single_index_slice(res, d, 0), axis=d), lo, axis=d))
            parts.append(res)
            if hi > 0:
                parts.append(repeat(expand_dims(_single_index_slice(res, d, res.shape[d] - 1), axis=d), hi, axis=d))
            res = concatenate(parts, axis=d)
        return res
    raise NotImplementedError(f"Pad mode '{mode}' is not supported. Only 'constant' and 'edge' modes are available.")


diff = Op("diff")


@diff.impl("hlo")
def _diff(a, n=1, axis=-1, prepend=None, append=None):
    from nkipy_b200.core.ops.elementwise import subtract

    nd = len(a.shape)
    ax = axis + nd if axis < 0 else axis
    parts = []
    if prepend is not None:
        parts.append(prepend)
    parts.append(a)
    if append is not None:
        parts.append(append)
    r = concatenate(parts, axis=ax) if len(parts) > 1 else a
    ctx = get_trace_context()
    for _ in range(n):
        t = _bt(r)
        size = t.shape[ax]
        s1, l1 = [0] * nd, list(t.shape)
        s1[ax] = 1
        s0, l0 = [0] * nd, list(t.shape)
        l0[ax] = size - 1
        r = subtract(NKIPyTensorRef(_slice_node(ctx, t, s1, l1)), NKIPyTensorRef(_slice_node(ctx, t, s0, l0)))
    return r


flip = Op("flip")


@flip.impl("hlo")
def _flip(x, axis=None):
    from nkipy_b200.core.ops.indexing import take

    nd = len(x.shape)
    if axis is None:
        axes = list(range(nd))
    elif isinstance(axis, int):
        axes = [axis + nd if axis < 0 else axis]
    else:
        axes = [a + nd if a < 0 else a for a in axis]
    r = x
    for a in axes:
        r = take(r, np.arange(r.shape[a] - 1, -1, -1, dtype=np.int32), axis=a)
    return r


tile = Op("tile")


@tile.impl("hlo")
def _tile(x, reps):
    reps = (reps,) if isinstance(reps, int) else tuple(reps)
    shape = tuple(x.shape)
    nd = len(shape)
    if len(reps) < nd:
        reps = (1,) * (nd - len(reps)) + reps
    elif len(reps) > nd:
        x = reshape(x, (1,) * (len(reps) - nd) + shape)
        shape = tuple(x.shape)
    if all(r == 1 for r in reps):
        return copy(x)
    inter = []
    for s in shape:
        inter += [1, s]
    r = reshape(x, tuple(inter))
    bshape = list(r.shape)
    for i, rep in enumerate(reps):
        bshape[2 * i] = rep
    r = broadcast_to(r, tuple(bshape))
    return reshape(r, tuple(rep * s for rep, s in zip(reps, shape)))


roll = Op("roll")


def _roll_axis(x, shift, axis):
    ctx = get_trace_context()
    t = _bt(x)
    size = t.shape[axis]
    nd = len(t.shape)
    shift = shift % size
    if shift == 0:
        return x if isinstance(x, NKIPyTensorRef) else NKIPyTensorRef(t)
    cut = size - shift
    s1, l1 = [0] * nd, list(t.shape)
    s1[axis] = cut
    s0, l0 = [0] * nd, list(t.shape)
    l0[axis] = cut
    tail = NKIPyTensorRef(_slice_node(ctx, t, s1, l1))
    head = NKIPyTensorRef(_slice_node(ctx, t, s0, l0))
    return concatenate([tail, head], axis=axis)


@roll.impl("hlo")
def _roll(x, shift, axis=None):
    shape = tuple(x.shape)
    nd = len(shape)
    if axis is None:
        flat = reshape(x, (int(np.prod(shape)),))
        return reshape(_roll_axis(flat, shift, 0), shape)
    if isinstance(shift, (list, tuple)):
        if not isinstance(axis, (list, tuple)):
            raise ValueError("If shift is a tuple, axis must also be a tuple")
        r = x
        for s, a in zip(shift, axis):
            r = _roll_axis(r, s, a + nd if a < 0 else a)
        return r
    return _roll_axis(x, shift, axis + nd if axis < 0 else axis)
