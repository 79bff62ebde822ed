"""Lazy elementwise expressions and their compilation into one ``ew`` launch.

A traced elementwise node (``add``, ``exponential``, ``compare``, ``select``,
``convert`` ... -- reference ``core/ops/binary.py``, ``unary.py``,
``indexing.py:20-110``, ``transform.py:480-500``) becomes an ``Expr`` node
instead of a kernel.  Leaves are strided views of materialised buffers,
scalar constants, or affine index functions (``iota``).  View ops applied to
an expression are pushed down to its leaves, so broadcast / transpose /
slice / reshape cost nothing.  When a value must exist in memory the
expression DAG is compiled to the register program of the ``ew`` kernel:
one launch per fused group, every leaf read once per output element.

Arithmetic follows the traced dtypes: fp32 registers for every float type
with a round-to-bf16/fp16 after each node of that type (NumPy/ml_dtypes
round per op), int32 registers for integers (narrow types wrapped after each
node), 0/1 for bools.
"""

import struct
from dataclasses import dataclass, field
from typing import List, Optional, Tuple

import ml_dtypes
import numpy as np

from nkipy_b200.planner import views as V

# dtype codes shared with libnkb (include/nkb.h enum nkb_dtype)
DT_CODES = {
    np.dtype(np.float32): 0,
    np.dtype(ml_dtypes.bfloat16): 1,
    np.dtype(np.float16): 2,
    np.dtype(np.int32): 3,
    np.dtype(np.uint32): 4,
    np.dtype(np.int8): 5,
    np.dtype(np.uint8): 6,
    np.dtype(np.bool_): 7,
    np.dtype(np.int16): 8,
    np.dtype(np.uint16): 9,
    np.dtype(ml_dtypes.float8_e4m3fn): 10,
    np.dtype(ml_dtypes.float8_e5m2): 11,
}


def dt_code(dt) -> int:
    dt = np.dtype(dt)
    if dt not in DT_CODES:
        raise NotImplementedError(f"dtype {dt} is not carried by the B200 path")
    return DT_CODES[dt]


def kind(dt) -> str:
    dt = np.dtype(dt)
    if dt == np.bool_:
        return "B"
    if dt.kind == "f" or dt in (np.dtype(ml_dtypes.bfloat16), np.dtype(ml_dtypes.float8_e4m3fn), np.dtype(ml_dtypes.float8_e5m2)):
        return "F"
    if dt.kind == "i":
        return "I"
    if dt.kind == "u":
        return "U"
    raise NotImplementedError(f"dtype {dt}")


# opcodes of k_elementwise.cu
OP = dict(
    NOP=0, LD=1, CF=2, CI=3, IOTA=4,
    FADD=10, FSUB=11, FMUL=12, FDIV=13, FPOW=14, FMAX=15, FMIN=16, FATAN2=17, FREM=18,
    FNEG=20, FABS=21, FEXP=22, FLOG=23, FSQRT=24, FRSQRT=25, FTANH=26, FSIN=27, FCOS=28, FFLOOR=29, FCEIL=30,
    FSIGN=31, RBF=32, RF16=33, FRCP=34,
    FEQ=40, FNE=41, FLT=42, FLE=43, FGT=44, FGE=45,
    IADD=50, ISUB=51, IMUL=52, IDIV=53, IMAX=54, IMIN=55, IAND=56, IOR=57, IXOR=58, IREM=59,
    ISHL=64, ISHR=65,
    INEG=60, IABS=61, INOT=62, ISIGN=63,
    IEQ=70, INE=71, ILT=72, ILE=73, IGT=74, IGE=75, ULT=76, ULE=77, UGT=78, UGE=79, UDIV=80, UMAX=81, UMIN=82, UREM=83,
    SEL=90,
    F2I=100, I2F=101, U2F=102, F2U=103, INZ=104, FNZ=105,
)

MAX_IN, MAX_RANK, MAX_INSTR, N_REGS = 8, 6, 64, 24

ELEMENTWISE_BINARY = {"add", "subtract", "multiply", "divide", "power", "maximum", "minimum", "and", "or", "xor",
                      "atan2", "remainder"}
ELEMENTWISE_UNARY = {"exponential", "log", "sqrt", "rsqrt", "tanh", "sine", "cosine", "floor", "ceil", "sign", "abs",
                     "negate", "not", "convert", "copy"}
ELEMENTWISE = ELEMENTWISE_BINARY | ELEMENTWISE_UNARY | {"compare", "select"}


@dataclass(eq=False)
class Expr:
    kind: str  # "leaf" | "const" | "affine" | "op"
    shape: Tuple[int, ...]
    dtype: np.dtype
    view: Optional[V.View] = None  # leaf
    value: object = None  # const
    offset: int = 0  # affine
    coefs: Tuple[int, ...] = ()  # affine
    op: str = ""  # op
    attrs: dict = field(default_factory=dict)
    args: List["Expr"] = field(default_factory=list)

    def leaves(self):
        seen, out = set(), []

        def walk(e):
            if id(e) in seen:
                return
            seen.add(id(e))
            if e.kind == "leaf":
                out.append(e)
            for a in e.args:
                walk(a)

        walk(self)
        return out

    def n_nodes(self):
        seen = set()

        def walk(e):
            if id(e) in seen:
                return
            seen.add(id(e))
            for a in e.args:
                walk(a)

        walk(self)
        return len(seen)


def leaf(view: V.View) -> Expr:
    return Expr("leaf", tuple(view.shape), np.dtype(view.dtype), view=view)


def const(value, dtype, shape=()) -> Expr:
    return Expr("const", tuple(shape), np.dtype(dtype), value=value)


def iota(shape, dtype, dim) -> Expr:
    coefs = [0] * len(shape)
    coefs[dim] = 1
    return Expr("affine", tuple(shape), np.dtype(dtype), offset=0, coefs=tuple(coefs))


def op(name, args, shape, dtype, attrs=None) -> Expr:
    return Expr("op", tuple(shape), np.dtype(dtype), op=name, args=list(args), attrs=dict(attrs or {}))


# ---------------------------------------------------------------------------
# view transforms pushed down to the leaves
# ---------------------------------------------------------------------------
def transform(e: Expr, new_shape, fn) -> Optional[Expr]:
    """Apply an index transform to every leaf.

    ``fn(offset, strides) -> (offset, strides) | None`` maps an affine index
    function over ``e.shape`` to one over ``new_shape``.
    """
    memo = {}

    def go(x: Expr) -> Optional[Expr]:
        if id(x) in memo:
            return memo[id(x)]
        if x.kind == "const":
            r = Expr("const", tuple(new_shape), x.dtype, value=x.value)
        elif x.kind == "leaf":
            t = fn(x.view.offset, x.view.strides)
            if t is None:
                return None
            r = Expr("leaf", tuple(new_shape), x.dtype, view=x.view.with_(offset=t[0], shape=tuple(new_shape), strides=t[1]))
        elif x.kind == "affine":
            t = fn(x.offset, x.coefs)
            if t is None:
                return None
            r = Expr("affine", tuple(new_shape), x.dtype, offset=t[0], coefs=t[1])
        else:
            args = []
            for a in x.args:
                ta = go(a)
                if ta is None:
                    return None
                args.append(ta)
            r = Expr("op", tuple(new_shape), x.dtype, op=x.op, args=args, attrs=x.attrs)
        memo[id(x)] = r
        return r

    return go(e)


def t_broadcast(e, new_shape, bdims):
    old = e.shape
    return transform(e, new_shape, lambda off, st: (off, V.broadcast_strides(old, st, new_shape, bdims)))


def t_transpose(e, perm):
    new_shape = tuple(e.shape[p] for p in perm)
    return transform(e, new_shape, lambda off, st: (off, V.transpose_strides(st, perm)))


def t_slice(e, starts, limits, steps):
    new_shape = tuple((hi - lo + s - 1) // s for lo, hi, s in zip(starts, limits, steps))
    return transform(e, new_shape, lambda off, st: V.slice_view(off, st, starts, steps))


def t_reshape(e, new_shape):
    old = e.shape

    def fn(off, st):
        ns = V.reshape_strides(old, st, new_shape)
        return None if ns is None else (off, ns)

    return transform(e, new_shape, fn)


# ---------------------------------------------------------------------------
# compilation to the ew register program
# ---------------------------------------------------------------------------
class TooBig(Exception):
    """The group exceeds the kernel's input/register/instruction budget."""


def _f32_bits(x) -> int:
    return struct.unpack("<I", struct.pack("<f", float(x)))[0]


def _i32_bits(x) -> int:
    return int(x) & 0xFFFFFFFF


def _narrow(prog, reg, dt):
    dt = np.dtype(dt)
    if dt in (np.dtype(np.int8), np.dtype(np.int16)):
        sh = 32 - 8 * dt.itemsize
        t = prog.tmp_const_int(sh)
        prog.emit("ISHL", reg, reg, t)
        prog.emit("ISHR", reg, reg, t)
        prog.release(t)
    elif dt in (np.dtype(np.uint8), np.dtype(np.uint16)):
        t = prog.tmp_const_int((1 << (8 * dt.itemsize)) - 1)
        prog.emit("IAND", reg, reg, t)
        prog.release(t)


def _round_float(prog, reg, dt):
    """Round the value just written to ``reg`` to a narrow float type.

    Folded into the producing instruction (its round field) when that
    instruction wrote ``reg``; otherwise an explicit RBF/RF16.
    """
    dt = np.dtype(dt)
    code = 1 if dt == np.dtype(ml_dtypes.bfloat16) else (2 if dt == np.dtype(np.float16) else 0)
    if not code:
        return
    last = prog.instrs[-1] if prog.instrs else None
    if last is not None and last[1] == reg and last[6] == 0 and last[0] not in (OP["LD"], OP["CF"], OP["CI"]):
        prog.instrs[-1] = last[:6] + (code,) + last[7:]
    else:
        prog.emit("RBF" if code == 1 else "RF16", reg, reg)


class _Prog:
    def __init__(self):
        self.instrs = []
        self.free = list(range(N_REGS - 1, -1, -1))

    def alloc(self):
        if not self.free:
            raise TooBig("registers")
        return self.free.pop()

    def release(self, r):
        self.free.append(r)

    def emit(self, name, dst, a=0, b=0, c=0, imm=0, bimm=0):
        if len(self.instrs) >= MAX_INSTR:
            raise TooBig("instructions")
        self.instrs.append((OP[name], dst, a, b, c, imm, 0, bimm))

    def tmp_const_int(self, v):
        r = self.alloc()
        self.emit("CI", r, imm=_i32_bits(v))
        return r


_FBIN = {"add": "FADD", "subtract": "FSUB", "multiply": "FMUL", "divide": "FDIV", "power": "FPOW", "maximum": "FMAX",
         "minimum": "FMIN", "atan2": "FATAN2", "remainder": "FREM"}
_IBIN = {"add": "IADD", "subtract": "ISUB", "multiply": "IMUL", "divide": "IDIV", "maximum": "IMAX", "minimum": "IMIN",
         "and": "IAND", "or": "IOR", "xor": "IXOR", "remainder": "IREM"}
_UBIN = dict(_IBIN, divide="UDIV", maximum="UMAX", minimum="UMIN", remainder="UREM")
_FUN = {"exponential": "FEXP", "log": "FLOG", "sqrt": "FSQRT", "rsqrt": "FRSQRT", "tanh": "FTANH", "sine": "FSIN",
        "cosine": "FCOS", "floor": "FFLOOR", "ceil": "FCEIL", "sign": "FSIGN", "abs": "FABS", "negate": "FNEG"}
_FCMP = {"EQ": "FEQ", "NE": "FNE", "LT": "FLT", "LE": "FLE", "GT": "FGT", "GE": "FGE"}
_ICMP = {"EQ": "IEQ", "NE": "INE", "LT": "ILT", "LE": "ILE", "GT": "IGT", "GE": "IGE"}
_UCMP = {"EQ": "IEQ", "NE": "INE", "LT": "ULT", "LE": "ULE", "GT": "UGT", "GE": "UGE"}


@dataclass
class CompiledEw:
    ints: List[int]
    in_views: List[V.View]
    n_instr: int


def compile_ew(expr: Expr, out: V.View) -> CompiledEw:
    """Program + launch geometry writing ``expr`` into view ``out``."""
    if tuple(out.shape) != tuple(expr.shape):
        raise ValueError(f"ew output shape {out.shape} != expression shape {expr.shape}")
    shape = tuple(int(s) for s in expr.shape) or (1,)
    # inputs: unique leaf views
    inputs: List[V.View] = []
    leaf_slot = {}
    for lf in expr.leaves():
        v = lf.view
        key = (v.buf, v.offset, tuple(v.strides), np.dtype(v.dtype).str)
        if key not in leaf_slot:
            leaf_slot[key] = len(inputs)
            inputs.append(v)
    if len(inputs) > MAX_IN:
        raise TooBig("inputs")
    # affine leaves join the axis collapsing as extra stride sets
    affines = []
    seen = set()

    def collect(e):
        if id(e) in seen:
            return
        seen.add(id(e))
        if e.kind == "affine":
            affines.append(e)
        for a in e.args:
            collect(a)

    collect(expr)
    full = lambda st: tuple(st) if st else (0,)  # noqa: E731
    sets = [full(out.strides)] + [full(v.strides) for v in inputs] + [full(a.coefs) for a in affines]
    cshape, csets = V.collapse(shape if expr.shape else (1,), sets)
    if len(cshape) > MAX_RANK:
        raise TooBig("rank")
    rank = len(cshape)
    out_st = csets[0]
    in_st = csets[1 : 1 + len(inputs)]
    aff_st = {id(a): csets[1 + len(inputs) + i] for i, a in enumerate(affines)}

    prog = _Prog()
    uses = {}

    def count(e):
        uses[id(e)] = uses.get(id(e), 0) + 1
        if uses[id(e)] == 1:
            for a in e.args:
                count(a)

    count(expr)
    reg_of = {}

    def value(e) -> int:
        if id(e) in reg_of:
            return reg_of[id(e)]
        r = gen(e)
        reg_of[id(e)] = r
        return r

    def done(e):
        uses[id(e)] -= 1
        if uses[id(e)] == 0 and id(e) in reg_of:
            prog.release(reg_of[id(e)])

    def gen(e) -> int:
        k = kind(e.dtype)
        if e.kind == "leaf":
            v = e.view
            key = (v.buf, v.offset, tuple(v.strides), np.dtype(v.dtype).str)
            r = prog.alloc()
            prog.emit("LD", r, leaf_slot[key])
            return r
        if e.kind == "const":
            r = prog.alloc()
            if k == "F":
                val = np.float32(e.value)
                if np.dtype(e.dtype) != np.float32:
                    val = np.float32(np.array(val).astype(e.dtype).astype(np.float32))
                prog.emit("CF", r, imm=_f32_bits(val))
            elif k == "B":
                prog.emit("CI", r, imm=1 if bool(e.value) else 0)
            else:
                prog.emit("CI", r, imm=_i32_bits(int(e.value)))
            return r
        if e.kind == "affine":
            st = aff_st[id(e)]
            r = prog.alloc()
            prog.emit("CI", r, imm=_i32_bits(e.offset))
            t = prog.alloc()
            for d, c in enumerate(st):
                if c == 0:
                    continue
                prog.emit("IOTA", t, d)
                if c != 1:
                    cr = prog.tmp_const_int(c)
                    prog.emit("IMUL", t, t, cr)
                    prog.release(cr)
                prog.emit("IADD", r, r, t)
            prog.release(t)
            if k == "F":
                prog.emit("I2F", r, r)
                _round_float(prog, r, e.dtype)
            return r
        # op node
        name = e.op
        args = e.args
        if name == "copy" or (name == "convert" and np.dtype(args[0].dtype) == np.dtype(e.dtype)):
            a = value(args[0])
            r = prog.alloc()
            prog.emit("IOR", r, a, a)  # register move
            done(args[0])
            return r
        if (name == "divide" and len(args) == 2 and k == "F" and args[0].kind == "const"
                and kind(args[1].dtype) == "F" and np.float32(args[0].value) == np.float32(1.0)):
            # 1 / x: the correctly rounded reciprocal, the same value as the division
            a = value(args[1])
            r = prog.alloc()
            prog.emit("FRCP", r, a)
            _round_float(prog, r, e.dtype)
            for x in e.args:
                done(x)
            return r
        imm_b = None
        if name in ELEMENTWISE_BINARY and len(args) == 2:
            if args[1].kind != "const" and args[0].kind == "const" and name in ("add", "multiply", "maximum", "minimum", "and", "or", "xor"):
                args = [args[1], args[0]]
            if args[1].kind == "const":
                imm_b = _imm_bits(args[1])
        regs = [value(a) for a in (args if imm_b is None else args[:1])]
        if imm_b is not None:
            regs.append(0)
        r = prog.alloc()
        if name == "convert":
            src = kind(args[0].dtype)
            a = regs[0]
            if src == "F" and k == "F":
                prog.emit("IOR", r, a, a)
                _round_float(prog, r, e.dtype)
            elif src == "F" and k == "I":
                prog.emit("F2I", r, a)
                _narrow(prog, r, e.dtype)
            elif src == "F" and k == "U":
                prog.emit("F2U", r, a)
                _narrow(prog, r, e.dtype)
            elif src == "F" and k == "B":
                prog.emit("FNZ", r, a)
            elif src in ("I", "B") and k == "F":
                prog.emit("I2F", r, a)
                _round_float(prog, r, e.dtype)
            elif src == "U" and k == "F":
                prog.emit("U2F", r, a)
                _round_float(prog, r, e.dtype)
            elif k == "B":
                prog.emit("INZ", r, a)
            else:
                prog.emit("IOR", r, a, a)
                _narrow(prog, r, e.dtype)
        elif name == "compare":
            ck = kind(args[0].dtype)
            table = _FCMP if ck == "F" else (_UCMP if ck == "U" else _ICMP)
            prog.emit(table[e.attrs["comparison_direction"]], r, regs[0], regs[1])
        elif name == "select":
            prog.emit("SEL", r, regs[0], regs[1], regs[2])
        elif name in ELEMENTWISE_BINARY:
            bi = dict(imm=imm_b, bimm=1) if imm_b is not None else {}
            if k == "F":
                if name not in _FBIN:
                    raise NotImplementedError(f"float {name}")
                prog.emit(_FBIN[name], r, regs[0], regs[1], **bi)
                _round_float(prog, r, e.dtype)
            elif k == "B":
                prog.emit(_IBIN[name], r, regs[0], regs[1], **bi)
            else:
                table = _UBIN if k == "U" else _IBIN
                if name not in table:
                    raise NotImplementedError(f"integer {name}")
                prog.emit(table[name], r, regs[0], regs[1], **bi)
                _narrow(prog, r, e.dtype)
        elif name == "not":
            if k == "B":
                one = prog.tmp_const_int(1)
                prog.emit("IXOR", r, regs[0], one)
                prog.release(one)
            else:
                prog.emit("INOT", r, regs[0])
                _narrow(prog, r, e.dtype)
        elif name in _FUN:
            if k == "F":
                prog.emit(_FUN[name], r, regs[0])
                _round_float(prog, r, e.dtype)
            elif name == "negate":
                prog.emit("INEG", r, regs[0])
                _narrow(prog, r, e.dtype)
            elif name == "abs":
                prog.emit("IABS" if k == "I" else "IOR", r, regs[0], regs[0])
            elif name == "sign":
                prog.emit("ISIGN", r, regs[0]) if k == "I" else prog.emit("INZ", r, regs[0])
            else:
                raise NotImplementedError(f"integer {name}")
        else:
            raise NotImplementedError(f"elementwise op {name}")
        for a in e.args:
            done(a)
        return r

    def _imm_bits(c):
        kc = kind(c.dtype)
        if kc == "F":
            val = np.float32(c.value)
            if np.dtype(c.dtype) != np.float32:
                val = np.float32(np.array(val).astype(c.dtype).astype(np.float32))
            return _f32_bits(val)
        if kc == "B":
            return 1 if bool(c.value) else 0
        return _i32_bits(int(c.value))

    out_reg = value(expr)
    ints = [len(inputs), rank, len(prog.instrs), dt_code(out.dtype), out_reg]
    contig = int(
        rank == 1 and out_st[0] == 1 and all(s[0] in (0, 1) for s in in_st)
    )
    n = int(np.prod(cshape))
    ints += [contig, n]
    ints += list(cshape)
    ints += [int(out.offset)] + list(out_st)
    for v, st in zip(inputs, in_st):
        ints += [dt_code(v.dtype), int(v.offset)] + list(st)
    for (o, d, a, b, c, imm, rnd, bimm) in prog.instrs:
        ints += [o, d, a, b, c, imm, rnd, bimm]
    return CompiledEw(ints=ints, in_views=inputs, n_instr=len(prog.instrs))
