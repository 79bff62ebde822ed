"""Strided views: how a traced tensor sits in a device buffer.

Every device buffer is dense row-major (the reference's layout,
``hlo.py:162-166``: ``minor_to_major = reversed(range(rank))``).  A value of the
graph is either materialised as ``View(buffer, offset, shape, strides)`` --
element offsets and strides, stride 0 for broadcast axes -- or still lazy.
``reshape``/``transpose``/``slice``/``broadcast`` of a materialised value are
folded into a new view whenever the result is still affine in the index
(no copy and no kernel); ``reshape_strides`` is the no-copy reshape test.
"""

from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np


def dense_strides(shape) -> Tuple[int, ...]:
    out, s = [], 1
    for d in reversed(shape):
        out.append(s)
        s *= int(d)
    return tuple(reversed(out))


@dataclass(frozen=True)
class View:
    buf: int  # plan buffer id
    offset: int  # element offset
    shape: Tuple[int, ...]
    strides: Tuple[int, ...]
    dtype: np.dtype

    @property
    def size(self) -> int:
        return int(np.prod(self.shape)) if self.shape else 1

    def is_dense(self) -> bool:
        """Row-major contiguous (size-1 axes ignored)."""
        want = dense_strides(self.shape)
        return all(s == 1 or a == b for s, a, b in zip(self.shape, self.strides, want))

    def with_(self, **kw) -> "View":
        d = dict(buf=self.buf, offset=self.offset, shape=self.shape, strides=self.strides, dtype=self.dtype)
        d.update(kw)
        return View(**d)


def reshape_strides(shape, strides, new_shape) -> Optional[Tuple[int, ...]]:
    """Strides for viewing (shape, strides) as new_shape without a copy, or None.

    Axes are grouped so that each group of old axes and the matching group of
    new axes have the same element count; inside a group the old axes must be
    mutually contiguous (stride[i] == stride[i+1] * shape[i+1], size-1 axes
    skipped), then the new axes of the group get strides from the group's
    innermost stride.
    """
    shape = [int(s) for s in shape]
    new_shape = [int(s) for s in new_shape]
    if int(np.prod(shape)) != int(np.prod(new_shape)):
        return None
    if int(np.prod(new_shape)) == 0:
        return dense_strides(new_shape)
    old = [(s, st) for s, st in zip(shape, strides) if s != 1]
    out = [0] * len(new_shape)
    oi, ni = 0, 0
    n_old, n_new = len(old), len(new_shape)
    while ni < n_new:
        if new_shape[ni] == 1:
            out[ni] = 0
            ni += 1
            continue
        if oi >= n_old:
            return None
        # grow groups until the products match
        o_end, n_end = oi + 1, ni + 1
        po, pn = old[oi][0], new_shape[ni]
        while po != pn:
            if po < pn:
                if o_end >= n_old:
                    return None
                po *= old[o_end][0]
                o_end += 1
            else:
                if n_end >= n_new:
                    return None
                pn *= new_shape[n_end]
                n_end += 1
        for k in range(oi, o_end - 1):
            if old[k][1] != old[k + 1][1] * old[k + 1][0]:
                return None
        st = old[o_end - 1][1]
        for k in range(n_end - 1, ni - 1, -1):
            if new_shape[k] == 1:
                out[k] = 0
                continue
            out[k] = st
            st *= new_shape[k]
        oi, ni = o_end, n_end
    return tuple(out)


def broadcast_strides(shape, strides, new_shape, bdims) -> Tuple[int, ...]:
    out = [0] * len(new_shape)
    for i, d in enumerate(bdims):
        if int(shape[i]) == int(new_shape[d]) and int(shape[i]) != 1:
            out[d] = strides[i]
    return tuple(out)


def transpose_strides(strides, perm) -> Tuple[int, ...]:
    return tuple(strides[p] for p in perm)


def slice_view(offset, strides, starts, steps):
    off = offset + sum(int(s) * int(st) for s, st in zip(starts, strides))
    return off, tuple(int(st) * int(k) for st, k in zip(strides, steps))


def collapse(shape, stride_sets):
    """Merge adjacent axes that are contiguous for every operand.

    ``stride_sets`` is a list of stride tuples (output first).  Returns the
    collapsed shape and stride sets; size-1 axes are dropped (rank >= 1).
    """
    shape = list(shape)
    keep = [i for i, s in enumerate(shape) if s != 1]
    if not keep:
        return (1,), [tuple([0]) for _ in stride_sets]
    shp = [shape[i] for i in keep]
    sts = [[st[i] for i in keep] for st in stride_sets]
    i = len(shp) - 1
    while i > 0:
        ok = all(st[i - 1] == st[i] * shp[i] for st in sts)
        if ok:
            shp[i - 1] *= shp[i]
            for st in sts:
                st[i - 1] = st[i]
                del st[i]
            del shp[i]
        i -= 1
    return tuple(shp), [tuple(st) for st in sts]
