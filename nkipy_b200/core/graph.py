"""Traced tensor graph: the IR that the B200 planner consumes.

The node vocabulary and attribute names are the reference's HLO opcode set
(``nkipy/core/backend/hlo.py:288-404`` for the containers,
``hlo.py:1538-1585`` for ``build_op``), so a graph traced here lists the same
ops, in the same order, as the reference tracer produces for the same kernel
body.  There is no protobuf emission: the graph is handed to
``nkipy_b200.planner`` instead of an external compiler.

Dtype promotion follows the reference's table (``hlo.py:1062-1358``), restated
here as rules over (kind, width) instead of an enumerated table; the rules are
checked entry by entry against a fixture dumped from the reference.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple, Union

import ml_dtypes
import numpy as np

from nkipy_b200.core import backend as _backend

bfloat16 = np.dtype(ml_dtypes.bfloat16)

# ---------------------------------------------------------------------------
# Containers
# ---------------------------------------------------------------------------


@dataclass(eq=False)
class TraceOp:
    """One graph node: an opcode applied to operand tensors."""

    op_name: str
    operands: List["TraceTensor"]
    result_shape: Tuple[int, ...]
    result_dtype: Any
    attributes: Dict[str, Any] = field(default_factory=dict)
    source_location: Optional[Tuple[str, int]] = None
    id: Optional[int] = None


@dataclass(eq=False)
class TraceTensor:
    """A value in the graph: a kernel parameter or the result of a node."""

    shape: Tuple[int, ...]
    dtype: Any
    source_op: Optional[TraceOp] = None
    is_parameter: bool = False
    parameter_id: Optional[int] = None
    name: str = ""
    id: Optional[int] = None


@dataclass
class TensorPlaceholder:
    name: str
    shape: Tuple[int, ...]
    dtype: Any


@dataclass(frozen=True)
class AliasInfo:
    """An output that must be written back into an input buffer.

    Same fields as the reference's ``AliasInfo`` (``hlo.py:320-332``).
    """

    output_index: int
    param_index: int
    param_name: str
    is_user_returned: bool


class TraceGraph:
    """Parameters, nodes in trace order, results and aliases of one kernel."""

    def __init__(self, name: str = "main") -> None:
        self.name = name
        self.parameters: List[TraceTensor] = []
        self.operations: List[TraceOp] = []
        self.results: List[TraceTensor] = []
        self.aliases: List[AliasInfo] = []
        self._next_id = 0

    @property
    def input_output_alias(self) -> Dict[int, int]:
        return {a.output_index: a.param_index for a in self.aliases}

    @property
    def auto_aliased_indices(self) -> set:
        return {a.output_index for a in self.aliases if not a.is_user_returned}

    @property
    def inputs(self) -> List[TensorPlaceholder]:
        return [TensorPlaceholder(p.name, tuple(p.shape), np.dtype(p.dtype)) for p in self.parameters]

    @property
    def outputs(self) -> List[TensorPlaceholder]:
        # A boolean result is carried as uint8 bytes, as the reference does
        # (hlo.py:370-379).
        out = []
        for r in self.results:
            dt = np.dtype(np.uint8) if np.dtype(r.dtype) == np.bool_ else np.dtype(r.dtype)
            out.append(TensorPlaceholder(r.name, tuple(r.shape), dt))
        return out

    def add_parameter(self, shape, dtype, name: str = "") -> TraceTensor:
        t = TraceTensor(
            shape=tuple(int(s) for s in shape),
            dtype=np.dtype(dtype),
            is_parameter=True,
            parameter_id=len(self.parameters),
            name=name,
        )
        self.parameters.append(t)
        return t

    def add_operation(self, op: TraceOp) -> TraceTensor:
        op.id = self._next_id
        self._next_id += 1
        self.operations.append(op)
        return TraceTensor(shape=tuple(op.result_shape), dtype=op.result_dtype, source_op=op, id=op.id)

    def set_results(self, results) -> None:
        self.results = list(results) if isinstance(results, (list, tuple)) else [results]

    # -- introspection used by the planner, the plan cache and the tests ----
    def op_names(self) -> List[str]:
        return [op.op_name for op in self.operations]

    def signature(self) -> str:
        """Deterministic text form of the graph (hash input for the plan cache)."""
        ids = {}
        for p in self.parameters:
            ids[id(p)] = f"p{p.parameter_id}"
        lines = [f"graph {self.name}"]
        for p in self.parameters:
            lines.append(f"param {p.parameter_id} {p.name} {tuple(p.shape)} {np.dtype(p.dtype).name}")
        res_by_op = {}
        for op in self.operations:
            operands = []
            for t in op.operands:
                if t.is_parameter:
                    operands.append(f"p{t.parameter_id}")
                else:
                    operands.append(f"%{t.id}")
            attrs = []
            for k in sorted(op.attributes):
                v = op.attributes[k]
                if isinstance(v, np.ndarray):
                    import hashlib

                    v = "nd:" + hashlib.sha256(np.ascontiguousarray(v).tobytes()).hexdigest()[:16] + str(v.shape) + v.dtype.name
                attrs.append(f"{k}={v}")
            lines.append(
                f"%{op.id} = {op.op_name}({','.join(operands)}) {tuple(op.result_shape)} "
                f"{np.dtype(op.result_dtype).name} {';'.join(attrs)}"
            )
        for i, r in enumerate(self.results):
            ref = f"p{r.parameter_id}" if r.is_parameter else f"%{r.id}"
            lines.append(f"result {i} {r.name} {ref}")
        for a in self.aliases:
            lines.append(f"alias {a}")
        return "\n".join(lines)


# Reference-compatible names (``hlo.py:288-340``).
HLOOp = TraceOp
HLOTensor = TraceTensor
HLOModule = TraceGraph


# ---------------------------------------------------------------------------
# Trace context
# ---------------------------------------------------------------------------


class TraceContext:
    """Builds nodes into a ``TraceGraph`` (reference: ``HLOTraceContext``)."""

    backend_name = "hlo"

    def __init__(self, module: TraceGraph) -> None:
        self.module = module
        self.current_source_location = None

    def set_source_location(self, location) -> None:
        self.current_source_location = location

    def get_source_location(self):
        return self.current_source_location

    def build_op(self, op_name, operands, result_shape, result_dtype, attributes=None, source_location=None):
        if isinstance(result_shape, list):
            result_shape = tuple(result_shape)
        op = TraceOp(
            op_name=op_name,
            operands=list(operands),
            result_shape=tuple(int(s) for s in result_shape),
            result_dtype=np.dtype(result_dtype),
            attributes=dict(attributes or {}),
            source_location=source_location or self.current_source_location,
        )
        return self.module.add_operation(op)


HLOTraceContext = TraceContext


def get_trace_context() -> TraceContext:
    ctx = _backend.active_context()
    if not isinstance(ctx, TraceContext):
        raise RuntimeError("No trace context is active.")
    return ctx


get_hlo_context = get_trace_context


# ---------------------------------------------------------------------------
# Dtype promotion
# ---------------------------------------------------------------------------


class _WeakInt:
    """Type key of a Python ``int`` operand (defers to the other operand)."""


class _WeakFloat:
    """Type key of a Python ``float`` operand (defers to float operands)."""


_F8 = {
    ml_dtypes.float8_e5m2,
    ml_dtypes.float8_e4m3fn,
    ml_dtypes.float8_e4m3,
}
_SIGNED = {np.int8: 8, np.int16: 16, np.int32: 32, np.int64: 64}
_UNSIGNED = {np.uint8: 8, np.uint16: 16, np.uint32: 32, np.uint64: 64}
_SIGNED_BY_WIDTH = {8: np.int8, 16: np.int16, 32: np.int32, 64: np.int64}
_UNSIGNED_BY_WIDTH = {8: np.uint8, 16: np.uint16, 32: np.uint32, 64: np.uint64}
_FLOAT_WIDE = {np.float16, np.float32, ml_dtypes.bfloat16}


def _type_key(val):
    if isinstance(val, bool):
        return np.bool_
    if isinstance(val, int):
        return _WeakInt
    if isinstance(val, float):
        return _WeakFloat
    if isinstance(val, (np.bool_, np.integer, np.floating)):
        return type(val)
    dt = getattr(val, "dtype", None)
    if dt is not None:
        if isinstance(dt, np.dtype):
            return dt.type
        if isinstance(dt, type):
            return dt
        try:
            return np.dtype(dt).type
        except (TypeError, ValueError):
            pass
    raise ValueError(f"Unsupported or unrecognized type: {type(val)}")


def _is_int(t):
    return t in _SIGNED or t in _UNSIGNED


def _promote_keys(a, b):
    """Result type key for two operand type keys, or None when undefined."""
    if a is np.float64 or b is np.float64:
        raise TypeError(
            "Unsupported dtype: float64. Use .astype(dtype) to convert to a supported type."
        )
    if a is b:
        return None if a in (_WeakInt, _WeakFloat) else a
    for x, y in ((a, b), (b, a)):
        # bool defers to everything; with a weak scalar it becomes int32/float32
        if x is np.bool_:
            if y is _WeakInt:
                return np.int32
            if y is _WeakFloat:
                return np.float32
            return y
    for x, y in ((a, b), (b, a)):
        # weak int defers to every strong numeric type
        if x is _WeakInt and y is not _WeakFloat:
            return y
        # weak float defers to floats; with an integer it gives float32
        if x is _WeakFloat and y is not _WeakInt:
            return np.float32 if _is_int(y) else y
    if a in (_WeakInt, _WeakFloat) and b in (_WeakInt, _WeakFloat):
        return None
    # float8 variants: defer to ints, lose to wider floats, never mix
    if a in _F8 or b in _F8:
        if a in _F8 and b in _F8:
            return None
        f8, other = (a, b) if a in _F8 else (b, a)
        if _is_int(other):
            return f8
        if other in _FLOAT_WIDE:
            return other
        return None
    a_int, b_int = _is_int(a), _is_int(b)
    if a_int and b_int:
        if a in _SIGNED and b in _SIGNED:
            return _SIGNED_BY_WIDTH[max(_SIGNED[a], _SIGNED[b])]
        if a in _UNSIGNED and b in _UNSIGNED:
            return _UNSIGNED_BY_WIDTH[max(_UNSIGNED[a], _UNSIGNED[b])]
        s, u = (a, b) if a in _SIGNED else (b, a)
        sw, uw = _SIGNED[s], _UNSIGNED[u]
        if uw < sw:
            return s
        if 2 * uw <= 64:
            return _SIGNED_BY_WIDTH[max(sw, 2 * uw)]
        return np.float32
    if a_int and b in _FLOAT_WIDE:
        return b
    if b_int and a in _FLOAT_WIDE:
        return a
    if a in _FLOAT_WIDE and b in _FLOAT_WIDE:
        # any mix of two distinct 16/32-bit floats lands on float32
        return np.float32
    return None


def _key_name(t):
    if t is _WeakInt:
        return "weak_int"
    if t is _WeakFloat:
        return "weak_float"
    return np.dtype(t).name


def find_common_type(x, y) -> np.dtype:
    """Common dtype of two operands (tensors, arrays or Python scalars)."""
    ka, kb = _type_key(x), _type_key(y)
    res = _promote_keys(ka, kb)
    if res is None:
        raise TypeError(
            f"No implicit dtype promotion path for {_key_name(ka)} and {_key_name(kb)}."
            " Use .astype(dtype) explicitly."
        )
    return np.dtype(res)


find_common_type_hlo = find_common_type


def scalar_dtype(scalar) -> np.dtype:
    """Strong dtype that a scalar constant is materialised with."""
    if isinstance(scalar, (bool, np.bool_)):
        return np.dtype(np.bool_)
    if isinstance(scalar, (np.integer, np.floating)):
        if isinstance(scalar, np.float64):
            raise ValueError("float64 is not supported; use .astype(np.float32) explicitly.")
        if isinstance(scalar, np.int64):
            return np.dtype(np.int32)
        if isinstance(scalar, np.uint64):
            return np.dtype(np.uint32)
        return scalar.dtype
    if isinstance(scalar, int):
        return np.dtype(np.int32)
    return np.dtype(np.float32)


# ---------------------------------------------------------------------------
# Constants and broadcasting
# ---------------------------------------------------------------------------


def as_graph_tensor(ctx: TraceContext, value, dtype) -> TraceTensor:
    """Scalar / ndarray / tensor -> graph tensor (scalars become ``constant``)."""
    if isinstance(value, TraceTensor):
        return value
    if np.isscalar(value):
        return ctx.module.add_operation(
            TraceOp("constant", [], (), np.dtype(dtype), {"value": float(value)})
        )
    if isinstance(value, np.ndarray):
        arr = value.astype(dtype) if value.dtype != np.dtype(dtype) else value
        return ctx.module.add_operation(TraceOp("constant", [], arr.shape, np.dtype(dtype), {"value": arr}))
    raise ValueError(f"Cannot convert {type(value)} to a graph tensor")


as_hlo_tensor = as_graph_tensor


def broadcast_to_shape(ctx: TraceContext, x: TraceTensor, target_shape) -> TraceTensor:
    """Numpy-rule broadcast of ``x`` to ``target_shape``.

    Emits the same node sequence as the reference (``hlo.py:1458-1506``):
    a ``reshape`` that prepends missing axes, a ``reshape`` that drops the
    size-1 axes being expanded, then one ``broadcast``.
    """
    target_shape = tuple(target_shape)
    if tuple(x.shape) == target_shape:
        return x
    missing = len(target_shape) - len(x.shape)
    if missing > 0:
        x = ctx.build_op("reshape", [x], (1,) * missing + tuple(x.shape), x.dtype)
    kept = []
    for d, (src, tgt) in enumerate(zip(x.shape, target_shape)):
        if src == tgt:
            kept.append(d)
        elif src != 1:
            raise ValueError(f"Cannot broadcast dimension {d} of size {src} to size {tgt}")
    squeezed = tuple(x.shape[d] for d in kept)
    if squeezed != tuple(x.shape):
        x = ctx.build_op("reshape", [x], squeezed, x.dtype)
    return ctx.build_op("broadcast", [x], target_shape, x.dtype, {"broadcast_dimensions": kept})


broadcast_to_shape_hlo = broadcast_to_shape


def broadcast_pair(ctx: TraceContext, x: TraceTensor, y: TraceTensor):
    if tuple(x.shape) == tuple(y.shape):
        return x, y
    target = tuple(np.broadcast_shapes(tuple(x.shape), tuple(y.shape)))
    if tuple(x.shape) != target:
        x = broadcast_to_shape(ctx, x, target)
    if tuple(y.shape) != target:
        y = broadcast_to_shape(ctx, y, target)
    return x, y


broadcast_operands_hlo = broadcast_pair
