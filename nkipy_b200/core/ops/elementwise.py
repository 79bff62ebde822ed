"""Elementwise ops: binary arithmetic, comparisons, logical ops and unary math.

Node emission follows the reference (``core/ops/binary.py:21-240``,
``core/ops/unary.py:14-306``): promote, turn scalars into ``constant``s,
broadcast with ``reshape``+``broadcast``, insert ``convert``s, then one node
with the HLO opcode (``add``, ``exponential``, ``compare`` + direction, ...).
Composite ops (``square``, ``reciprocal``, ``rint``, ``log1p`` ...) are built
from the primitive ones exactly as the reference decomposes them.
"""

import numpy as np

from nkipy_b200.core.graph import as_graph_tensor, broadcast_pair, find_common_type, get_trace_context
from nkipy_b200.core.ops._registry import Op
from nkipy_b200.core.tensor import NKIPyTensorRef

_BINARY_OPCODES = {
    "add": "add",
    "subtract": "subtract",
    "multiply": "multiply",
    "divide": "divide",
    "power": "power",
    "maximum": "maximum",
    "minimum": "minimum",
    "bitwise_and": "and",
    "bitwise_or": "or",
    "bitwise_xor": "xor",
}

_COMPARE_DIRECTIONS = {
    "equal": "EQ",
    "not_equal": "NE",
    "less": "LT",
    "less_equal": "LE",
    "greater": "GT",
    "greater_equal": "GE",
}

_UNARY_OPCODES = {
    "abs": "abs",
    "exp": "exponential",
    "log": "log",
    "sqrt": "sqrt",
    "sin": "sine",
    "cos": "cosine",
    "tanh": "tanh",
    "negative": "negate",
    "ceil": "ceil",
    "floor": "floor",
    "sign": "sign",
    "invert": "not",
    "bitwise_not": "not",
}


def _operand(ctx, v, dtype):
    return v.backend_tensor if isinstance(v, NKIPyTensorRef) else as_graph_tensor(ctx, v, dtype)


def _binary(opcode, x, y, dtype=None):
    ctx = get_trace_context()
    promoted = find_common_type(x, y)
    out_dtype = np.dtype(dtype) if dtype is not None else promoted
    a = _operand(ctx, x, promoted)
    b = _operand(ctx, y, promoted)
    a, b = broadcast_pair(ctx, a, b)
    if np.dtype(a.dtype) != out_dtype:
        a = ctx.build_op("convert", [a], a.shape, out_dtype)
    if np.dtype(b.dtype) != out_dtype:
        b = ctx.build_op("convert", [b], b.shape, out_dtype)
    return NKIPyTensorRef(ctx.build_op(opcode, [a, b], a.shape, out_dtype))


def _compare(direction, x, y):
    ctx = get_trace_context()
    promoted = find_common_type(x, y)
    a = _operand(ctx, x, promoted)
    b = _operand(ctx, y, promoted)
    if np.dtype(a.dtype) != promoted:
        a = ctx.build_op("convert", [a], a.shape, promoted)
    if np.dtype(b.dtype) != promoted:
        b = ctx.build_op("convert", [b], b.shape, promoted)
    a, b = broadcast_pair(ctx, a, b)
    return NKIPyTensorRef(
        ctx.build_op("compare", [a, b], a.shape, np.bool_, {"comparison_direction": direction})
    )


def _nonzero_mask(ctx, t):
    zero = as_graph_tensor(ctx, 0, t.dtype)
    if t.shape:
        zero = ctx.build_op("broadcast", [zero], t.shape, t.dtype, {"broadcast_dimensions": []})
    return ctx.build_op("compare", [t, zero], t.shape, np.bool_, {"comparison_direction": "NE"})


def _logical(opcode, x, y):
    ctx = get_trace_context()
    promoted = find_common_type(x, y)
    a = _operand(ctx, x, promoted)
    b = _operand(ctx, y, promoted)
    a, b = broadcast_pair(ctx, a, b)
    ma = _nonzero_mask(ctx, a)
    mb = _nonzero_mask(ctx, b)
    return NKIPyTensorRef(ctx.build_op(opcode, [ma, mb], a.shape, np.bool_))


def _unary(opcode, x):
    ctx = get_trace_context()
    t = x.backend_tensor if isinstance(x, NKIPyTensorRef) else x
    return NKIPyTensorRef(ctx.build_op(opcode, [t], t.shape, t.dtype))


def _make_binary(name):
    op = Op(name)
    opcode = _BINARY_OPCODES[name]

    @op.impl("hlo")
    def _impl(x, y, out=None, dtype=None):
        return _binary(opcode, x, y, dtype)

    return op


def _make_compare(name):
    op = Op(name)
    direction = _COMPARE_DIRECTIONS[name]

    @op.impl("hlo")
    def _impl(x, y, out=None, dtype=None):
        return _compare(direction, x, y)

    return op


def _make_logical(name, opcode):
    op = Op(name)

    @op.impl("hlo")
    def _impl(x, y, out=None, dtype=None):
        return _logical(opcode, x, y)

    return op


def _make_unary(name):
    op = Op(name)
    opcode = _UNARY_OPCODES[name]

    @op.impl("hlo")
    def _impl(x, out=None, dtype=None):
        return _unary(opcode, x)

    return op


add = _make_binary("add")
subtract = _make_binary("subtract")
multiply = _make_binary("multiply")
divide = _make_binary("divide")
power = _make_binary("power")
maximum = _make_binary("maximum")
minimum = _make_binary("minimum")
bitwise_and = _make_binary("bitwise_and")
bitwise_or = _make_binary("bitwise_or")
bitwise_xor = _make_binary("bitwise_xor")

equal = _make_compare("equal")
not_equal = _make_compare("not_equal")
greater = _make_compare("greater")
greater_equal = _make_compare("greater_equal")
less = _make_compare("less")
less_equal = _make_compare("less_equal")

logical_and = _make_logical("logical_and", "and")
logical_or = _make_logical("logical_or", "or")
logical_xor = _make_logical("logical_xor", "xor")

abs = _make_unary("abs")  # noqa: A001 - mirrors numpy naming
exp = _make_unary("exp")
log = _make_unary("log")
sqrt = _make_unary("sqrt")
negative = _make_unary("negative")
sin = _make_unary("sin")
cos = _make_unary("cos")
tanh = _make_unary("tanh")
ceil = _make_unary("ceil")
floor = _make_unary("floor")
sign = _make_unary("sign")
invert = _make_unary("invert")
bitwise_not = _make_unary("bitwise_not")

arctan = Op("arctan")


@arctan.impl("hlo")
def _arctan(x, out=None, dtype=None):
    ctx = get_trace_context()
    t = x.backend_tensor
    one = as_graph_tensor(ctx, 1.0, t.dtype)
    if t.shape:
        one = ctx.build_op("broadcast", [one], t.shape, t.dtype, {"broadcast_dimensions": []})
    return NKIPyTensorRef(ctx.build_op("atan2", [t, one], t.shape, t.dtype))


# -- composites (same decompositions as the reference) ----------------------
logaddexp = Op("logaddexp")


@logaddexp.impl("hlo")
def _logaddexp(x, y):
    m = maximum(x, y)
    return add(m, log(add(exp(subtract(x, m)), exp(subtract(y, m)))))


remainder = Op("remainder")


@remainder.impl("hlo")
def _remainder(x, y):
    return subtract(x, multiply(y, floor(divide(x, y))))


floor_divide = Op("floor_divide")


@floor_divide.impl("hlo")
def _floor_divide(x, y):
    return floor(divide(x, y))


reciprocal = Op("reciprocal")


@reciprocal.impl("hlo")
def _reciprocal(x, out=None, dtype=None):
    return divide(1.0, x)


square = Op("square")


@square.impl("hlo")
def _square(x, out=None, dtype=None):
    return multiply(x, x)


tan = Op("tan")


@tan.impl("hlo")
def _tan(x, out=None, dtype=None):
    return divide(sin(x), cos(x))


rint = Op("rint")


@rint.impl("hlo")
def _rint(x, out=None, dtype=None):
    from nkipy_b200.core.ops.indexing import where

    fl = floor(x)
    frac = subtract(x, fl)
    up = add(fl, 1.0)
    gt_half = greater(frac, 0.5)
    odd = not_equal(subtract(fl, multiply(floor(divide(fl, 2.0)), 2.0)), 0.0)
    tie_odd = logical_and(equal(frac, 0.5), odd)
    return where(tie_odd, up, where(gt_half, up, fl))


trunc = Op("trunc")


@trunc.impl("hlo")
def _trunc(x, out=None, dtype=None):
    from nkipy_b200.core.ops.indexing import where

    return where(greater_equal(x, 0), floor(x), ceil(x))


logical_not = Op("logical_not")


@logical_not.impl("hlo")
def _logical_not(x, out=None, dtype=None):
    return equal(x, 0)


clip = Op("clip")


@clip.impl("hlo")
def _clip(x, a_min=None, a_max=None, out=None):
    r = x
    if a_min is not None:
        r = maximum(r, a_min)
    if a_max is not None:
        r = minimum(r, a_max)
    return r


log1p = Op("log1p")


@log1p.impl("hlo")
def _log1p(x, out=None, dtype=None):
    return log(add(x, 1.0))


log2 = Op("log2")


@log2.impl("hlo")
def _log2(x, out=None, dtype=None):
    return divide(log(x), float(np.log(2.0)))


expm1 = Op("expm1")


@expm1.impl("hlo")
def _expm1(x, out=None, dtype=None):
    return subtract(exp(x), 1.0)


round_ = Op("round")


@round_.impl("hlo")
def _round(x, decimals=0, out=None):
    if decimals == 0:
        return rint(x)
    scale = float(10**decimals)
    return divide(rint(multiply(x, scale)), scale)


isnan = Op("isnan")


@isnan.impl("hlo")
def _isnan(x, out=None, dtype=None):
    return not_equal(x, x)


isfinite = Op("isfinite")


@isfinite.impl("hlo")
def _isfinite(x, out=None, dtype=None):
    return equal(subtract(x, x), 0.0)
