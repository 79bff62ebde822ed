"""The launch plan: what ``nkb_plan_load`` consumes (it replaces a NEFF).

A plan lists the io table (byte sizes of inputs in parameter order and of
outputs in result order), constant buffers (uploaded once after load), a
scratch arena with the offsets of every intermediate, and the ordered
kernel launches.  ``to_text`` writes the line format parsed by
``nkb_runtime.cu``; ``digest`` hashes it for the plan cache.
"""

import hashlib
from dataclasses import dataclass, field
from typing import List, Tuple

import numpy as np

ALIGN = 256


@dataclass
class BufDecl:
    kind: str  # "in" | "out" | "const" | "tmp" | "symm"
    index: int  # io / const index (tmp, symm: -1)
    nbytes: int
    offset: int = 0  # arena offset (tmp) or offset in the symmetric region (symm)


@dataclass
class StepRec:
    kernel: str
    bufs: List[Tuple[int, int]]  # (buffer id, byte offset)
    ints: List[int] = field(default_factory=list)
    floats: List[float] = field(default_factory=list)
    note: str = ""


@dataclass
class IoSpec:
    name: str
    shape: Tuple[int, ...]
    dtype: np.dtype

    @property
    def nbytes(self) -> int:
        return int(np.prod(self.shape, dtype=np.int64)) * np.dtype(self.dtype).itemsize if self.shape else np.dtype(self.dtype).itemsize


@dataclass
class Plan:
    name: str
    inputs: List[IoSpec]
    outputs: List[IoSpec]
    consts: List[np.ndarray]
    buffers: List[BufDecl]
    steps: List[StepRec]
    scratch: int = 0
    aliases: list = field(default_factory=list)  # (output index, input index)
    needs_comm: bool = False
    symm: int = 0  # bytes of the symmetric region the "symm" buffers need

    def to_text(self) -> str:
        lines = ["NKBPLAN 1", f"name {self.name or 'kernel'}"]
        lines.append(f"inputs {len(self.inputs)}")
        for i, s in enumerate(self.inputs):
            lines.append(f"input {i} {s.nbytes}")
        lines.append(f"outputs {len(self.outputs)}")
        for i, s in enumerate(self.outputs):
            lines.append(f"output {i} {s.nbytes}")
        lines.append(f"consts {len(self.consts)}")
        for i, c in enumerate(self.consts):
            lines.append(f"const {i} {c.nbytes}")
        lines.append(f"scratch {self.scratch}")
        if self.symm:
            lines.append(f"symm {self.symm}")
        lines.append(f"buffers {len(self.buffers)}")
        for i, b in enumerate(self.buffers):
            if b.kind in ("tmp", "symm"):
                lines.append(f"buffer {i} {b.kind} {b.offset} {b.nbytes}")
            else:
                lines.append(f"buffer {i} {b.kind} {b.index}")
        lines.append(f"steps {len(self.steps)}")
        for s in self.steps:
            parts = ["step", s.kernel, str(len(s.bufs))]
            for bid, off in s.bufs:
                parts += [str(bid), str(int(off))]
            parts.append(str(len(s.ints)))
            parts += [str(int(v)) for v in s.ints]
            parts.append(str(len(s.floats)))
            parts += [repr(float(v)) for v in s.floats]
            lines.append(" ".join(parts))
        lines.append("end")
        return "\n".join(lines) + "\n"

    def digest(self) -> str:
        h = hashlib.sha256(self.to_text().encode())
        for c in self.consts:
            h.update(np.ascontiguousarray(c).tobytes())
        return h.hexdigest()[:16]

    def kernel_counts(self):
        out = {}
        for s in self.steps:
            out[s.kernel] = out.get(s.kernel, 0) + 1
        return out

    def summary(self) -> str:
        rows = [f"plan {self.name}: {len(self.steps)} launches, scratch {self.scratch / 2**20:.1f} MiB"]
        for s in self.steps:
            rows.append(f"  {s.kernel:<14} {s.note}")
        return "\n".join(rows)


SYMM_ALIGN = 4096


def pack_symmetric(buffers: List[BufDecl]) -> int:
    """Give every "symm" buffer its own offset in the symmetric region (they are
    few and large: the operands of all-reduces); returns the region size."""
    top = 0
    for b in buffers:
        if b.kind == "symm":
            b.offset = top
            top += (b.nbytes + SYMM_ALIGN - 1) // SYMM_ALIGN * SYMM_ALIGN
    return top


def pack_arena(buffers: List[BufDecl], lifetimes) -> int:
    """Assign arena offsets to tmp buffers whose lifetimes overlap disjointly.

    ``lifetimes[i] = (first_step, last_step)``.  Greedy by size: each buffer
    takes the lowest offset not used by a placed buffer that is live at the
    same time.
    """
    order = sorted(
        [i for i, b in enumerate(buffers) if b.kind == "tmp"], key=lambda i: -buffers[i].nbytes
    )
    placed = []
    top = 0
    for i in order:
        size = (buffers[i].nbytes + ALIGN - 1) // ALIGN * ALIGN
        lo, hi = lifetimes.get(i, (0, 0))
        busy = sorted(
            (buffers[j].offset, buffers[j].offset + (buffers[j].nbytes + ALIGN - 1) // ALIGN * ALIGN)
            for j in placed
            if not (lifetimes.get(j, (0, 0))[1] < lo or lifetimes.get(j, (0, 0))[0] > hi)
        )
        off = 0
        for a, b in busy:
            if off + size <= a:
                break
            off = max(off, b)
        buffers[i].offset = off
        placed.append(i)
        top = max(top, off + size)
    return top
