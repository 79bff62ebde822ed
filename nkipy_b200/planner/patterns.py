"""Recognisers that map decomposed NumPy compositions back onto fused kernels.

The reference never emits ``softmax`` or ``rms_norm`` nodes (their ops are
declared without an implementation, ``core/ops/nn.py:12-160``): a kernel body
writes them as NumPy compositions, and the tracer records the primitive
nodes plus reshape/broadcast noise.  Each recogniser here walks one such
composition backwards from its last node and, when every interior value is
used only inside the composition, claims the nodes for one fused launch:

* row softmax      reduce-max, subtract, exponential, reduce-add, divide
                   (``tests/kernels/softmax.py:7-10``), optional bf16<->f32
                   converts around it (``qwen3_embedding/kernels/softmax.py``);
* RMSNorm          square, mean (reduce-add / N), + eps, sqrt, divide, * w,
                   optional residual add in front and dtype converts
                   (``qwen3_embedding/kernels/rmsnorm.py:4-16``);
* argmax / argmin  reduce-max, compare, float iota, select, reduce-min,
                   convert to int32 (``core/ops/reduce.py:227-311``);
* attention        dot(q, k^T) -> / sqrt(d) -> + causal mask constant ->
                   softmax -> dot(., v), with the transposes and the GQA
                   ``np.repeat`` of k/v feeding it
                   (``qwen3_embedding/kernels/attention.py:75-95``).
"""

import hashlib
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import ml_dtypes
import numpy as np

NOISE = ("reshape", "broadcast")


def tkey(t):
    return ("p", t.parameter_id) if t.is_parameter else ("o", t.id)


class GraphIndex:
    def __init__(self, graph):
        self.graph = graph
        self.consumers: Dict[tuple, List] = {}
        for op in graph.operations:
            for t in op.operands:
                self.consumers.setdefault(tkey(t), []).append(op)
        self.results = {tkey(r) for r in graph.results}

    def uses(self, t) -> int:
        return len(self.consumers.get(tkey(t), [])) + (1 if tkey(t) in self.results else 0)

    @staticmethod
    def producer(t):
        return None if t.is_parameter else t.source_op


def strip(t, ops: list, allowed=NOISE):
    """Follow reshape/broadcast producers back to the underlying value."""
    while True:
        p = GraphIndex.producer(t)
        if p is None or p.op_name not in allowed:
            return t
        ops.append(p)
        t = p.operands[0]


def _is_float(dt) -> bool:
    from nkipy_b200.planner.ewprog import kind

    return kind(dt) == "F"


def strip_copy(t, ops: list):
    """Skip ``copy`` nodes and float -> float32 ``convert`` nodes."""
    while True:
        p = GraphIndex.producer(t)
        if p is None:
            return t
        if p.op_name == "copy" or (
            p.op_name == "convert" and np.dtype(p.result_dtype) == np.float32 and _is_float(p.operands[0].dtype)
        ):
            ops.append(p)
            t = p.operands[0]
            continue
        return t


def scalar_const(t, ops: list):
    base = strip(t, ops)
    p = GraphIndex.producer(base)
    if p is None or p.op_name != "constant":
        return None
    v = p.attributes.get("value")
    if isinstance(v, np.ndarray):
        if v.size != 1:
            return None
        v = v.reshape(()).item()
    ops.append(p)
    return float(v)


def is_row_bcast(t, full_shape, ops: list):
    """t is a (rows,)-vector broadcast back over the last axis of full_shape."""
    p = GraphIndex.producer(t)
    if p is None or p.op_name != "broadcast" or tuple(p.result_shape) != tuple(full_shape):
        return None
    n = len(full_shape)
    if list(p.attributes.get("broadcast_dimensions", [])) != list(range(n - 1)):
        return None
    ops.append(p)
    return strip(p.operands[0], ops)


def last_axis_reduce(t, computation, ops: list):
    p = GraphIndex.producer(t)
    if p is None or p.op_name != "reduce" or p.attributes.get("computation") != computation:
        return None
    x = p.operands[0]
    if list(p.attributes.get("dimensions", [])) != [len(x.shape) - 1]:
        return None
    ops.append(p)
    ops.append(GraphIndex.producer(p.operands[1]))  # init constant
    return x


@dataclass
class Claim:
    kind: str
    root: object  # the op whose result the fused kernel produces
    interior: List = field(default_factory=list)
    params: dict = field(default_factory=dict)


def _exclusive(gi: GraphIndex, ops, root) -> bool:
    """Every value produced inside (except the root's) is consumed only inside."""
    inside = {id(o) for o in ops if o is not None} | {id(root)}
    for o in ops:
        if o is None or o is root:
            continue
        t_key = ("o", o.id)
        if t_key in gi.results:
            return False
        for c in gi.consumers.get(t_key, []):
            if id(c) not in inside:
                return False
    return True


def match_softmax(gi: GraphIndex, div_op, allow_bf16=False) -> Optional[Claim]:
    """Row softmax in fp32; ``allow_bf16`` also takes the all-bf16 form (the
    Qwen3 ``softmax_kernel``), for callers that evaluate it inside a fused
    attention kernel in fp32."""
    if div_op.op_name != "divide" or len(div_op.result_shape) < 1:
        return None
    shape = tuple(div_op.result_shape)
    ops = []
    e, bs = div_op.operands
    pe = GraphIndex.producer(e)
    if pe is None or pe.op_name != "exponential":
        return None
    ops.append(pe)
    sub = GraphIndex.producer(pe.operands[0])
    if sub is None or sub.op_name != "subtract":
        return None
    ops.append(sub)
    x, bm = sub.operands
    s_base = is_row_bcast(bs, shape, ops)
    if s_base is None:
        return None
    e2 = last_axis_reduce(s_base, "add", ops)
    if e2 is None or tkey(e2) != tkey(e):
        return None
    m_base = is_row_bcast(bm, shape, ops)
    if m_base is None:
        return None
    x2 = last_axis_reduce(m_base, "maximum", ops)
    if x2 is None or tkey(x2) != tkey(x):
        return None
    ok_dt = np.dtype(div_op.result_dtype) == np.float32 or (allow_bf16 and str(np.dtype(div_op.result_dtype)) == "bfloat16")
    if not ok_dt or tuple(x.shape) != shape:
        return None
    if not _exclusive(gi, ops, div_op):
        return None
    # absorb a bf16 -> f32 convert feeding x, and an f32 -> bf16 convert after
    src = x
    px = GraphIndex.producer(x)
    if px is not None and px.op_name == "convert" and str(np.dtype(px.operands[0].dtype)) == "bfloat16" and gi.uses(
        x
    ) == 2:
        ops.append(px)
        src = px.operands[0]
    root = div_op
    out_dtype = np.dtype(np.float32)
    cons = gi.consumers.get(("o", div_op.id), [])
    if len(cons) == 1 and ("o", div_op.id) not in gi.results and cons[0].op_name == "convert" and str(
        np.dtype(cons[0].result_dtype)
    ) == "bfloat16":
        ops.append(div_op)
        root = cons[0]
        out_dtype = np.dtype(cons[0].result_dtype)
    return Claim("softmax", root, [o for o in ops if o is not None and o is not root], {"x": src, "out_dtype": out_dtype})


def match_rmsnorm(gi: GraphIndex, mul_op) -> Optional[Claim]:
    if mul_op.op_name != "multiply" or len(mul_op.result_shape) < 1:
        return None
    shape = tuple(mul_op.result_shape)
    cols = shape[-1]
    for zz, wb in (mul_op.operands, mul_op.operands[::-1]):
        ops = []
        pzz = GraphIndex.producer(zz)
        if pzz is None or pzz.op_name != "divide":
            continue
        ops.append(pzz)
        x32, qb = pzz.operands
        q = is_row_bcast(qb, shape, ops)
        if q is None:
            continue
        psq = GraphIndex.producer(q)
        if psq is None or psq.op_name != "sqrt":
            continue
        ops.append(psq)
        # ``(z + eps).astype(x.dtype)`` with x already fp32 traces as a copy
        pa = GraphIndex.producer(strip(psq.operands[0], ops, allowed=("copy",)))
        if pa is None or pa.op_name != "add":
            continue
        ops.append(pa)
        m, eb = pa.operands
        eps = scalar_const(eb, ops)
        if eps is None:
            continue
        pm = GraphIndex.producer(m)
        if pm is None or pm.op_name != "divide":
            continue
        ops.append(pm)
        s_keep, cb = pm.operands
        n = scalar_const(cb, ops)
        if n is None or int(round(n)) != cols:
            continue
        z = last_axis_reduce(strip(s_keep, ops), "add", ops)
        if z is None:
            continue
        pz = GraphIndex.producer(z)
        if pz is None or pz.op_name != "multiply" or tkey(pz.operands[0]) != tkey(pz.operands[1]) or tkey(
            pz.operands[0]
        ) != tkey(x32):
            continue
        ops.append(pz)
        # weight: a (cols,) vector broadcast along the rows
        pwb = GraphIndex.producer(wb)
        if pwb is None or pwb.op_name != "broadcast":
            continue
        bd = list(pwb.attributes["broadcast_dimensions"])
        src_shape = tuple(pwb.operands[0].shape)
        if not bd or bd[-1] != len(shape) - 1 or src_shape[-1] != cols or any(s_ != 1 for s_ in src_shape[:-1]):
            continue
        ops.append(pwb)
        w32 = strip(pwb.operands[0], ops)
        if tuple(w32.shape) != (cols,):
            continue
        w = strip_copy(w32, ops)
        if np.dtype(mul_op.result_dtype) != np.float32 or tuple(x32.shape) != shape:
            continue
        x = strip_copy(x32, ops)
        if not _exclusive(gi, ops, mul_op):
            continue
        # residual add in front of the norm
        res = None
        px = GraphIndex.producer(x)
        if px is not None and px.op_name == "add" and tuple(px.operands[0].shape) == shape and tuple(
            px.operands[1].shape
        ) == shape and np.dtype(px.operands[0].dtype) == np.dtype(px.operands[1].dtype) == np.dtype(px.result_dtype):
            res = px
        root = mul_op
        out_dtype = np.dtype(np.float32)
        cons = gi.consumers.get(("o", mul_op.id), [])
        if len(cons) == 1 and ("o", mul_op.id) not in gi.results and cons[0].op_name in ("convert", "copy"):
            ops.append(mul_op)
            root = cons[0]
            out_dtype = np.dtype(cons[0].result_dtype)
        if out_dtype != np.dtype(x.dtype):
            continue
        params = {"x": x, "w": w, "eps": eps, "out_dtype": out_dtype, "residual": None, "sum_needed": False}
        if res is None and root is not mul_op:
            rope = _rope_after_norm(gi, root, shape)
            if rope is not None:
                rops, params["rope"], cat = rope
                ops.append(root)
                ops += [o for o in rops if o is not cat]
                root = cat
        if res is not None:
            params["residual"] = (res.operands[0], res.operands[1])
            inside = {id(o) for o in ops if o is not None} | {id(root), id(mul_op)}
            params["sum_needed"] = tkey(x) in gi.results or any(
                id(c) not in inside for c in gi.consumers.get(tkey(x), [])
            )
            ops.append(res)
            params["sum_tensor"] = x
        return Claim("rmsnorm", root, [o for o in ops if o is not None and o is not root], params)
    return None


def _carried_axes(t, ops: list):
    """Follow reshape (unit axes only) and broadcast producers from ``t`` back to
    the underlying value.  Returns ``(base, axes)``: ``axes[i]`` is the axis of
    ``base`` that axis ``i`` of ``t`` runs along (None: broadcast or unit)."""
    p = GraphIndex.producer(t)
    shp = [int(d) for d in t.shape]
    if p is None or p.op_name not in ("reshape", "broadcast"):
        return t, [i if shp[i] != 1 else None for i in range(len(shp))]
    base, axes = _carried_axes(p.operands[0], ops)
    if base is None:
        return None, None
    ops.append(p)
    src = [int(d) for d in p.operands[0].shape]
    out = [None] * len(shp)
    if p.op_name == "broadcast":
        for i, d in enumerate(p.attributes["broadcast_dimensions"]):
            out[d] = axes[i] if src[i] == shp[d] else None
        return base, out
    src_nu = [(axes[i], src[i]) for i in range(len(src)) if src[i] != 1]
    dst_nu = [i for i in range(len(shp)) if shp[i] != 1]
    if [n for _, n in src_nu] != [shp[i] for i in dst_nu]:
        return None, None  # a reshape that merges or splits axes
    for (a, _), i in zip(src_nu, dst_nu):
        out[i] = a
    return base, out


def _table_row_gather(base):
    """``(table, index)`` when ``base`` (1, n) is row ``index`` of a 2-D table,
    gathered at run time (``tensor_apis.constant(cos)[start_pos]``)."""
    pg = GraphIndex.producer(base)
    if pg is None or pg.op_name != "gather" or len(base.shape) != 2 or int(base.shape[0]) != 1:
        return None
    a = pg.attributes
    tbl, idx = pg.operands
    if list(a.get("collapsed_slice_dims", [])) != [0] or list(a.get("start_index_map", [])) != [0]:
        return None
    if len(tbl.shape) != 2 or int(np.prod(idx.shape)) != 1 or np.dtype(idx.dtype).kind not in "iu":
        return None
    if list(a.get("slice_sizes", [])) != [1, int(tbl.shape[1])] or int(tbl.shape[1]) != int(base.shape[1]):
        return None
    return tbl, idx, pg


def _rope_after_norm(gi: GraphIndex, heads_op, shape):
    """The half-split rotation (rope.py:34-57) applied to the bf16 (B, S, H, hd)
    output of a per-head RMSNorm, every node bf16, with cos / sin either a row
    of a table gathered at a run-time position (decode) or an (S, hd/2) table
    read per token (prefill).  Returns (ops, params, concatenate op) or None."""
    if len(shape) != 4 or shape[3] not in (64, 128) or str(np.dtype(heads_op.result_dtype)) != "bfloat16":
        return None
    rot = _rotation_of(gi, heads_op)
    if rot is None:
        return None
    cat, rops, cos_b, sin_b = rot
    if any(str(np.dtype(o.result_dtype)) != "bfloat16" for o in rops):
        return None
    half = shape[3] // 2
    src = {}
    for m in (o for o in rops if o.op_name == "multiply"):
        for t in m.operands:
            if GraphIndex.producer(t) in rops:
                continue  # the half slice
            base, axes = _carried_axes(t, [])
            if base is None or _table_key(base) not in (_table_key(cos_b), _table_key(sin_b)):
                return None
            src.setdefault(_table_key(base), set()).add(tuple(axes))
    if len(src) != 2 or any(len(v) != 1 for v in src.values()):
        return None
    tables = {}
    for name, b in (("cos", cos_b), ("sin", sin_b)):
        bs = [int(d) for d in b.shape]
        last = len(bs) - 1
        if str(np.dtype(b.dtype)) != "bfloat16" or not bs or bs[last] != half:
            return None
        (axes,) = src[_table_key(b)]
        nonunit = {i for i, d in enumerate(bs) if d != 1}
        g = _table_row_gather(b)
        if g is not None:
            if list(axes) != [None, None, None, last]:
                return None
            tables[name] = {"table": g[0], "rows": int(g[0].shape[0]), "pos": g[1], "gather": g[2], "per_token": 0}
        elif axes[3] == last and axes[0] is None and axes[2] is None and axes[1] is not None \
                and bs[axes[1]] == shape[1] and nonunit <= {axes[1], last}:
            # an (S, hd/2) table (possibly with unit axes) read per token
            tables[name] = {"table": b, "rows": shape[1], "pos": None, "gather": None, "per_token": 1}
        elif list(axes) == [None, None, None, last] and nonunit <= {last}:
            tables[name] = {"table": b, "rows": 1, "pos": None, "gather": None, "per_token": 0}
        else:
            return None
    c, sn = tables["cos"], tables["sin"]
    if c["per_token"] != sn["per_token"] or (c["pos"] is None) != (sn["pos"] is None):
        return None
    if c["pos"] is not None and (tkey(c["pos"]) != tkey(sn["pos"]) or tuple(c["table"].shape) != tuple(sn["table"].shape)):
        return None
    params = {"cos": c["table"], "sin": sn["table"], "rows": c["rows"], "pos": c["pos"], "per_token": c["per_token"],
              "gathers": [g for g in (c["gather"], sn["gather"]) if g is not None]}
    return rops, params, cat


def absorb_rope_gathers(gi: GraphIndex, claims, taken: set):
    """A rotary-table row gathered at run time whose every use lies inside
    fused RMSNorm + rotation claims (which read the table at the position
    themselves): the gather and the reshape / broadcast views of its row are
    taken out of the graph."""
    for c in list(claims.values()):
        rope = c.params.get("rope") if c.kind == "rmsnorm" else None
        for g in (rope or {}).get("gathers", []):
            if id(g) in taken or ("o", g.id) in gi.results:
                continue
            chain, frontier, ok = [g], [g], True
            while frontier and ok:
                op = frontier.pop()
                for u in gi.consumers.get(("o", op.id), []):
                    if id(u) in taken:
                        continue
                    if u.op_name in ("reshape", "broadcast") and ("o", u.id) not in gi.results:
                        chain.append(u)
                        frontier.append(u)
                    else:
                        ok = False
            if ok:
                taken |= {id(o) for o in chain}


def match_argmax(gi: GraphIndex, cvt_op) -> Optional[Claim]:
    if cvt_op.op_name != "convert" or np.dtype(cvt_op.result_dtype) != np.int32:
        return None
    ops = []
    sel_t = last_axis_reduce(cvt_op.operands[0], "minimum", ops)
    if sel_t is None:
        return None
    psel = GraphIndex.producer(sel_t)
    if psel is None or psel.op_name != "select":
        return None
    ops.append(psel)
    mask, io, big = psel.operands
    pio = GraphIndex.producer(io)
    n = len(sel_t.shape)
    if pio is None or pio.op_name != "iota" or pio.attributes.get("iota_dimension") != n - 1:
        return None
    ops.append(pio)
    if scalar_const(big, ops) is None:
        return None
    pm = GraphIndex.producer(mask)
    if pm is None or pm.op_name != "compare" or pm.attributes.get("comparison_direction") != "EQ":
        return None
    ops.append(pm)
    x, bx = pm.operands
    ext = is_row_bcast(bx, tuple(x.shape), ops)
    if ext is None:
        return None
    pr = GraphIndex.producer(ext)
    if pr is None or pr.op_name != "reduce":
        return None
    comp = pr.attributes.get("computation")
    if comp not in ("maximum", "minimum"):
        return None
    x2 = last_axis_reduce(ext, comp, ops)
    if x2 is None or tkey(x2) != tkey(x):
        return None
    if not _exclusive(gi, ops, cvt_op):
        return None
    if np.dtype(x.dtype) not in (np.dtype(np.float32), np.dtype(np.float16), np.dtype(ml_dtypes.bfloat16)):
        return None  # the row kernel reads floats; other dtypes keep the generic lowering
    return Claim("argmax", cvt_op, [o for o in ops if o is not None], {"x": x, "is_max": comp == "maximum"})


def _trace_kv(t, ops: list):
    """Follow transposes (and one GQA repeat) back from an attention operand.

    Returns (source tensor, axis map, n_rep): operand axis i reads source axis
    amap[i]; when a repeat (broadcast of a new axis after the head axis +
    reshape merging it) is found, the head axis of the source is indexed by
    head // n_rep.
    """
    amap = list(range(len(t.shape)))
    cur = t
    while True:
        p = GraphIndex.producer(cur)
        if p is not None and p.op_name == "transpose":
            perm = list(p.attributes["permutation"])
            amap = [perm[a] for a in amap]
            ops.append(p)
            cur = p.operands[0]
            continue
        break
    n_rep = 1
    p = GraphIndex.producer(cur)
    if p is not None and p.op_name == "reshape":
        pb = GraphIndex.producer(p.operands[0])
        out_shape = tuple(p.result_shape)
        if pb is not None and pb.op_name == "broadcast" and len(out_shape) == 4:
            bshape = tuple(pb.result_shape)
            bd = list(pb.attributes["broadcast_dimensions"])
            src = pb.operands[0]
            # (B, S, Hkv, D) -> (B, S, Hkv, rep, D) -> (B, S, Hkv*rep, D)
            if (
                len(bshape) == 5
                and bd == [0, 1, 2, 4]
                and tuple(src.shape) == (bshape[0], bshape[1], bshape[2], bshape[4])
                and out_shape == (bshape[0], bshape[1], bshape[2] * bshape[3], bshape[4])
            ):
                n_rep = bshape[3]
                ops += [p, pb]
                cur = src
    return cur, amap, n_rep


def _is_causal_mask(arr, sq, skv):
    """True: causal with the queries at the end of the keys (query i sees keys
    up to i + skv - sq); "prefix": query i sees keys 0..i only, so keys from
    sq on are masked for every query (a cache prefill, ``mask[:S, :L]``);
    False: all zero; None: anything else."""
    a = np.asarray(arr).astype(np.float32)
    a = a.reshape(a.shape[-2:]) if a.size == sq * skv else None
    if a is None or a.shape != (sq, skv):
        return None
    rows = np.arange(sq)[:, None]
    cols = np.arange(skv)[None, :]
    for shift, kind in ((skv - sq, True), (0, "prefix")):
        upper = cols > rows + shift
        if np.all(a[~upper] == 0) and np.all(a[upper] <= -1000.0):
            return kind
    if np.all(a == 0):
        return False
    return None


def _const_array(t, ops: list):
    """The value of ``t`` when it is a constant or a slice of one."""
    p = GraphIndex.producer(t)
    if p is None:
        return None
    if p.op_name == "constant" and isinstance(p.attributes.get("value"), np.ndarray):
        ops.append(p)
        return np.asarray(p.attributes["value"])
    if p.op_name == "slice":
        v = _const_array(p.operands[0], ops)
        if v is None:
            return None
        a = p.attributes
        ops.append(p)
        return v[tuple(slice(int(b), int(e), int(st)) for b, e, st in
                       zip(a["start_indices"], a["limit_indices"], a["strides"]))]
    return None


def match_attention(gi: GraphIndex, dot2) -> Optional[Claim]:
    if dot2.op_name != "dot" or len(dot2.result_shape) != 4:
        return None
    at = dot2.attributes
    if at["lhs_batch_dimensions"] != [0, 1] or at["rhs_batch_dimensions"] != [0, 1]:
        return None
    if at["lhs_contracting_dimensions"] != [3] or at["rhs_contracting_dimensions"] != [2]:
        return None
    p_t, v_t = dot2.operands
    pp = GraphIndex.producer(p_t)
    if pp is None:
        return None
    div = GraphIndex.producer(pp.operands[0]) if pp.op_name == "convert" else pp
    if div is None or div.op_name != "divide":
        return None
    sm = match_softmax(gi, div, allow_bf16=True)
    if sm is None or sm.root is not pp:
        return None
    ops = [pp] + list(sm.interior)
    x = sm.params["x"]
    sq, skv = int(x.shape[2]), int(x.shape[3])
    causal = False
    kv_len = skv  # keys read: a prefix-causal mask masks keys from sq on
    pos = None  # decode: the run-time row of a causal mask table
    px = GraphIndex.producer(x)
    scaled = x
    if px is not None and px.op_name == "add":
        for a, m in (px.operands, px.operands[::-1]):
            tmp = []
            base = strip(m, tmp)
            cops = []
            val = _const_array(base, cops)
            if val is not None:
                c = _is_causal_mask(val, sq, skv)
                if c is not None:
                    causal = bool(c)
                    if c == "prefix":
                        kv_len = sq
                    ops += tmp + cops + [px]
                    scaled = a
                    break
            if sq == 1:
                got = _mask_row_at(base, skv, tmp)
                if got is not None:
                    pos = got
                    ops += tmp + [px]
                    scaled = a
                    break
        if scaled is x:
            return None
    scale = 1.0
    raw = _strip_float_converts(scaled, ops)
    ps = GraphIndex.producer(raw)
    if ps is not None and ps.op_name in ("divide", "multiply"):
        tmp = []
        c = scalar_const(ps.operands[1], tmp)
        if c is not None and c != 0:
            scale = 1.0 / c if ps.op_name == "divide" else c
            ops += tmp + [ps]
            raw = _strip_float_converts(ps.operands[0], ops)
    pr = GraphIndex.producer(raw)
    if pr is None or pr.op_name != "dot":
        return None
    a1 = pr.attributes
    if a1["lhs_batch_dimensions"] != [0, 1] or a1["rhs_batch_dimensions"] != [0, 1]:
        return None
    if a1["lhs_contracting_dimensions"] != [3] or a1["rhs_contracting_dimensions"] != [2]:
        return None
    ops.append(pr)
    q_t, kt_t = pr.operands
    for t in (q_t, kt_t, v_t):
        if str(np.dtype(t.dtype)) != "bfloat16":
            return None
    if str(np.dtype(dot2.result_dtype)) != "bfloat16" or str(np.dtype(x.dtype)) != "bfloat16":
        return None
    if not _exclusive(gi, ops, dot2):
        return None
    # operand paths: claimed only when they feed nothing else
    qops, kops, vops = [], [], []
    q_src, q_map, q_rep = _trace_kv(q_t, qops)
    k_src, k_map, k_rep = _trace_kv(kt_t, kops)
    v_src, v_map, v_rep = _trace_kv(v_t, vops)
    if q_rep != 1 or k_rep != v_rep:
        return None
    d = int(q_t.shape[3])
    if d not in (64, 128):
        return None
    path_ops = []
    for po in (qops, kops, vops):
        if po and _exclusive(gi, po + ops, dot2):
            path_ops += po
    if pos is not None and d != 128:
        return None
    params = dict(
        q=q_src, q_map=q_map, k=k_src, k_map=[k_map[0], k_map[1], k_map[3], k_map[2]], v=v_src, v_map=v_map,
        n_rep=k_rep, scale=scale, causal=causal, sq=sq, skv=skv, kv_len=kv_len, d=d, heads=int(q_t.shape[1]),
        batch=int(q_t.shape[0]), pos=pos,
    )
    if not path_ops:
        # the operand paths are shared: read the dot operands as they are
        params.update(q=q_t, q_map=[0, 1, 2, 3], k=kt_t, k_map=[0, 1, 3, 2], v=v_t, v_map=[0, 1, 2, 3], n_rep=1)
    return Claim("attention", dot2, ops + path_ops, params)


def _strip_float_converts(t, ops: list):
    """Skip float -> float ``convert`` nodes (the traced scale is computed in
    fp32 between a bf16 dot and a bf16 cast)."""
    while True:
        p = GraphIndex.producer(t)
        if p is None or p.op_name != "convert" or not (_is_float(p.result_dtype) and _is_float(p.operands[0].dtype)):
            return t
        ops.append(p)
        t = p.operands[0]


def _mask_row_at(base, skv, ops: list):
    """The index tensor ``pos`` when ``base`` is row ``pos`` of a constant causal
    mask table (0 up to the diagonal, large negative above), gathered at run
    time: the decode step's ``causal_mask[start_pos, :L]``
    (``examples/models/qwen3/kernels/attention.py:128-140``)."""
    pg = GraphIndex.producer(base)
    if pg is None or pg.op_name != "gather":
        return None
    a = pg.attributes
    if list(a.get("collapsed_slice_dims", [])) != [0] or list(a.get("start_index_map", [])) != [0]:
        return None
    tbl, idx = pg.operands
    if len(tbl.shape) != 2 or int(np.prod(idx.shape)) != 1 or np.dtype(idx.dtype).kind not in "iu":
        return None
    if list(a.get("slice_sizes", [])) != [1, skv]:
        return None
    local = [pg]
    src = tbl
    psl = GraphIndex.producer(src)
    if psl is not None and psl.op_name == "slice":
        sa = psl.attributes
        if list(sa["start_indices"]) != [0, 0] or set(sa["strides"]) != {1} or int(sa["limit_indices"][1]) != skv:
            return None
        local.append(psl)
        src = psl.operands[0]
    pc = GraphIndex.producer(src)
    if pc is None or pc.op_name != "constant" or not isinstance(pc.attributes.get("value"), np.ndarray):
        return None
    table = np.asarray(pc.attributes["value"])
    rows = int(tbl.shape[0])
    if table.ndim != 2 or table.shape[0] < rows or table.shape[1] < skv:
        return None
    if _is_causal_mask(table[:rows, :skv], rows, skv) is not True or rows != skv:
        return None
    ops += local + [pc]
    return idx


def _const_value(t):
    tmp = []
    return scalar_const(t, tmp), tmp


def _last_axis_half(t, which, ops):
    """t = slice of a dot result selecting its first (0) / second (1) half along the last axis."""
    p = GraphIndex.producer(t)
    if p is None or p.op_name != "slice":
        return None
    src = p.operands[0]
    n = len(src.shape)
    full = int(src.shape[-1])
    if full % 2:
        return None
    a = p.attributes
    want_start = [0] * (n - 1) + [which * full // 2]
    want_limit = list(src.shape[:-1]) + [(which + 1) * full // 2]
    if list(a["start_indices"]) != want_start or list(a["limit_indices"]) != want_limit or set(a["strides"]) != {1}:
        return None
    ops.append(p)
    return src


def match_swiglu_gemm(gi: GraphIndex, mul_op) -> Optional[Claim]:
    """gate, up = split(x @ W, 2, -1); silu(gate) * up  (``qwen3_embedding/kernels/ffn.py:4-46``)."""
    if mul_op.op_name != "multiply" or str(np.dtype(mul_op.result_dtype)) != "bfloat16":
        return None
    for a_t, u_t in (mul_op.operands, mul_op.operands[::-1]):
        ops = []
        d_up = _last_axis_half(u_t, 1, ops)
        if d_up is None:
            continue
        pa = GraphIndex.producer(a_t)
        if pa is None or pa.op_name != "multiply":
            continue
        ops.append(pa)
        for g_t, r_t in (pa.operands, pa.operands[::-1]):
            o2 = list(ops)
            d_g = _last_axis_half(g_t, 0, o2)
            if d_g is None or tkey(d_g) != tkey(d_up):
                continue
            pr = GraphIndex.producer(r_t)
            if pr is None or pr.op_name != "divide":
                continue
            one, t1 = _const_value(pr.operands[0])
            if one != 1.0:
                continue
            o2 += t1 + [pr]
            pd = GraphIndex.producer(pr.operands[1])
            if pd is None or pd.op_name != "add":
                continue
            o2.append(pd)
            ok = False
            for c_t, e_t in (pd.operands, pd.operands[::-1]):
                one2, t2 = _const_value(c_t)
                pe = GraphIndex.producer(e_t)
                if one2 == 1.0 and pe is not None and pe.op_name == "exponential":
                    pn = GraphIndex.producer(pe.operands[0])
                    if pn is not None and pn.op_name == "negate" and tkey(pn.operands[0]) == tkey(g_t):
                        o2 += t2 + [pe, pn]
                        ok = True
                        break
            if not ok:
                continue
            pdot = GraphIndex.producer(d_up)
            if pdot is None or pdot.op_name != "dot" or str(np.dtype(pdot.result_dtype)) != "bfloat16":
                continue
            o2.append(pdot)
            if not _exclusive(gi, o2, mul_op):
                continue
            return Claim("swiglu_gemm", mul_op, o2, {"dot": pdot, "gate": g_t, "up": u_t, "n_half": int(d_up.shape[-1]) // 2})
    return None


def _prod(op_name, t, ops, n_args=None):
    p = GraphIndex.producer(t)
    if p is None or p.op_name != op_name or (n_args is not None and len(p.operands) != n_args):
        return None
    ops.append(p)
    return p


def _elu1_of(t, ops):
    """t = select(x > 0, x + 1, exp(x)) with x = convert(src -> f32); returns src."""
    sel = _prod("select", t, ops)
    if sel is None:
        return None
    cond, a, b = sel.operands
    pc = _prod("compare", cond, ops)
    if pc is None or pc.attributes.get("comparison_direction") != "GT":
        return None
    x = pc.operands[0]
    if scalar_const(pc.operands[1], ops) != 0.0:
        return None
    pa = _prod("add", a, ops)
    pe = _prod("exponential", b, ops)
    if pa is None or pe is None or tkey(pa.operands[0]) != tkey(x) or tkey(pe.operands[0]) != tkey(x):
        return None
    if scalar_const(pa.operands[1], ops) != 1.0:
        return None
    pcv = GraphIndex.producer(x)
    if pcv is None or pcv.op_name != "convert":
        return None
    ops.append(pcv)
    return pcv.operands[0]


def _cumsum_of(t, ops):
    """t = cumsum(x, axis) as core/ops/reduce.py:320-385 traces it; returns x."""
    pt = _prod("transpose", t, ops)
    if pt is None:
        return None
    pr = _prod("reshape", pt.operands[0], ops)
    if pr is None:
        return None
    pd = _prod("dot", pr.operands[0], ops)
    if pd is None:
        return None
    tri = GraphIndex.producer(pd.operands[1])
    if tri is None or tri.op_name != "constant":
        return None
    val = np.asarray(tri.attributes.get("value"))
    if val.ndim != 2 or not np.array_equal(val, np.triu(np.ones_like(val))):
        return None
    ops.append(tri)
    pr2 = _prod("reshape", pd.operands[0], ops)
    if pr2 is None:
        return None
    pt2 = _prod("transpose", pr2.operands[0], ops)
    if pt2 is None or list(pt2.attributes["permutation"]) != list(pt.attributes["permutation"]):
        return None
    return pt2.operands[0]


def match_linear_attention(gi: GraphIndex, root) -> Optional[Claim]:
    """The chunked linear attention body of nkipy_b200/workloads.py (elu+1, causal, normalised)."""
    if root.op_name != "convert" or len(root.result_shape) != 4:
        return None
    ops = []
    rs = _prod("reshape", root.operands[0], ops)
    if rs is None:
        return None
    dv = _prod("divide", rs.operands[0], ops)
    if dv is None:
        return None
    num_t, den_b = dv.operands
    den_t = strip(den_b, ops)
    pnum = _prod("add", num_t, ops)
    pden = _prod("add", den_t, ops)
    if pnum is None or pden is None:
        return None
    # numerator: dot(Sm, V) + dot(Phi_q, State)
    d1 = _prod("dot", pnum.operands[0], ops)
    d2 = _prod("dot", pnum.operands[1], ops)
    if d1 is None or d2 is None:
        return None
    sm_t, vc_t = d1.operands
    phq_t, st_t = d2.operands
    pm = _prod("multiply", sm_t, ops)
    if pm is None:
        return None
    scores_t, mask_b = pm.operands
    tri = GraphIndex.producer(strip(mask_b, ops))
    if tri is None or tri.op_name != "constant":
        return None
    tv = np.asarray(tri.attributes.get("value"))
    if tv.ndim != 2 or not np.array_equal(tv, np.tril(np.ones_like(tv))):
        return None
    ops.append(tri)
    chunk = tv.shape[0]
    psc = _prod("dot", scores_t, ops)
    if psc is None or tkey(psc.operands[0]) != tkey(phq_t):
        return None
    ptk = _prod("transpose", psc.operands[1], ops)
    if ptk is None:
        return None
    phk_t = ptk.operands[0]
    # state = cumsum(KV) - KV, KV = Phi_k^T V
    pst = _prod("subtract", st_t, ops)
    if pst is None:
        return None
    pkv = _prod("dot", pst.operands[1], ops)
    if pkv is None or tkey(pkv.operands[1]) != tkey(vc_t):
        return None
    ptk2 = _prod("transpose", pkv.operands[0], ops)
    if ptk2 is None or tkey(ptk2.operands[0]) != tkey(phk_t):
        return None
    cs = _cumsum_of(pst.operands[0], ops)
    if cs is None or tkey(cs) != tkey(pst.operands[1]):
        return None
    # denominator: rowsum(Sm) + rowsum(Phi_q * zsum)
    r1 = last_axis_reduce(strip(pden.operands[0], ops), "add", ops)
    r2 = last_axis_reduce(strip(pden.operands[1], ops), "add", ops)
    if r1 is None or r2 is None or tkey(r1) != tkey(sm_t):
        return None
    pqz = _prod("multiply", r2, ops)
    if pqz is None or tkey(pqz.operands[0]) != tkey(phq_t):
        return None
    pz = _prod("subtract", strip(pqz.operands[1], ops), ops)
    if pz is None:
        return None
    ksum_t = pz.operands[1]
    csz = _cumsum_of(pz.operands[0], ops)
    if csz is None or tkey(csz) != tkey(ksum_t):
        return None
    pks = _prod("reshape", ksum_t, ops)
    if pks is None:
        return None
    pkr = GraphIndex.producer(pks.operands[0])
    if pkr is None or pkr.op_name != "reduce" or pkr.attributes.get("computation") != "add":
        return None
    ops += [pkr, GraphIndex.producer(pkr.operands[1])]
    if tkey(pkr.operands[0]) != tkey(phk_t):
        return None
    # feature maps and value convert
    pq_r = _prod("reshape", phq_t, ops)
    pk_r = _prod("reshape", phk_t, ops)
    pv_r = _prod("reshape", vc_t, ops)
    if pq_r is None or pk_r is None or pv_r is None:
        return None
    q_src = _elu1_of(pq_r.operands[0], ops)
    k_src = _elu1_of(pk_r.operands[0], ops)
    pvc = _prod("convert", pv_r.operands[0], ops)
    if q_src is None or k_src is None or pvc is None:
        return None
    v_src = pvc.operands[0]
    shape = tuple(root.result_shape)
    for t in (q_src, k_src, v_src):
        if tuple(t.shape) != shape or str(np.dtype(t.dtype)) != "bfloat16":
            return None
    if str(np.dtype(root.result_dtype)) != "bfloat16" or shape[3] != 128 or chunk != 64 or shape[2] % chunk:
        return None
    ops = [o for o in ops if o is not None]
    if not _exclusive(gi, ops, root):
        return None
    return Claim("linattn", root, ops, {"q": q_src, "k": k_src, "v": v_src, "shape": shape})


def match_residual_gemm(gi: GraphIndex, add_op) -> Optional[Claim]:
    """h + x @ W with the product used only by the add (the residual after the
    FFN down projection, ``qwen3_embedding/kernels/transformer_layer.py:60-83``):
    the add becomes the GEMM's epilogue."""
    if add_op.op_name != "add" or len(add_op.operands) != 2 or str(np.dtype(add_op.result_dtype)) != "bfloat16":
        return None
    for d_t, r_t in (add_op.operands, add_op.operands[::-1]):
        pd = GraphIndex.producer(d_t)
        if pd is None or pd.op_name != "dot" or str(np.dtype(pd.result_dtype)) != "bfloat16":
            continue
        if tuple(r_t.shape) != tuple(add_op.result_shape) or tuple(d_t.shape) != tuple(add_op.result_shape):
            continue
        if str(np.dtype(r_t.dtype)) != "bfloat16" or tkey(r_t) == tkey(d_t):
            continue
        if not _exclusive(gi, [pd], add_op):
            continue
        return Claim("residual_gemm", add_op, [pd], {"dot": pd, "res": r_t})
    return None


def _view_base(t, ops):
    """Strip reshape/broadcast ops (appending them to ops); the underlying tensor."""
    while True:
        p = GraphIndex.producer(t)
        if p is None or p.op_name not in ("reshape", "broadcast"):
            return t
        ops.append(p)
        t = p.operands[0]


def _last_axis_slice(op, n_axes):
    """(start, limit) of a slice that only narrows the last of n_axes axes, else None."""
    if op.op_name != "slice" or len(op.operands[0].shape) != n_axes:
        return None
    st, lim = list(op.attributes["start_indices"]), list(op.attributes["limit_indices"])
    strides = op.attributes.get("strides") or [1] * n_axes
    full = op.operands[0].shape
    if any(int(x) != 1 for x in strides):
        return None
    if any(st[i] != 0 or lim[i] != full[i] for i in range(n_axes - 1)):
        return None
    return int(st[-1]), int(lim[-1])


def _table_key(t):
    """Identity of a rotary table operand: a traced constant (a NumPy table
    becomes one constant node per use) by its value, anything else by tensor."""
    pc = GraphIndex.producer(t)
    if pc is not None and pc.op_name == "constant" and isinstance(pc.attributes.get("value"), np.ndarray):
        v = np.ascontiguousarray(pc.attributes["value"])
        return ("const", v.shape, str(v.dtype), hashlib.blake2b(v.tobytes(), digest_size=16).digest())
    return tkey(t)


def _rotation_of(gi: GraphIndex, heads_op):
    """heads_op's result (B, S, H, hd): the traced half-split rotation of
    rope.py:34-57, concatenate([x0 * cos - x1 * sin, x0 * sin + x1 * cos], -1)
    with x0, x1 its halves.  Returns (concat op, interior ops, cos, sin) or None."""
    hd = int(heads_op.result_shape[-1])
    half = hd // 2
    key = ("o", heads_op.id)
    users = gi.consumers.get(key, [])
    if len(users) != 2 or key in gi.results:
        return None
    halves = {}
    for u in users:
        rng = _last_axis_slice(u, 4)
        if rng == (0, half):
            halves[0] = u
        elif rng == (half, hd):
            halves[1] = u
    if len(halves) != 2:
        return None
    ops = [halves[0], halves[1]]
    prods = {}  # (half, base tensor key) -> (multiply op, base tensor)
    for i in (0, 1):
        mults = gi.consumers.get(("o", halves[i].id), [])
        if len(mults) != 2 or any(m.op_name != "multiply" for m in mults):
            return None
        for m in mults:
            a, b = m.operands
            other = b if tkey(a) == ("o", halves[i].id) else a
            base = _view_base(other, [])  # the table's reshape/broadcast views stay outside the claim
            ops.append(m)
            prods[(i, _table_key(base))] = (m, base)
    # lo = x0*cos - x1*sin and hi = x0*sin + x1*cos: find the subtract and the add
    outs = {}
    for (i, bk), (m, base) in prods.items():
        for c in gi.consumers.get(("o", m.id), []):
            if c.op_name in ("subtract", "add"):
                outs.setdefault(c.id, c)
    if len(outs) != 2:
        return None
    sub = next((c for c in outs.values() if c.op_name == "subtract"), None)
    add = next((c for c in outs.values() if c.op_name == "add"), None)
    if sub is None or add is None:
        return None
    def src(c, j):
        p = GraphIndex.producer(c.operands[j])
        for (i, bk), (m, base) in prods.items():
            if p is m:
                return i, bk, base
        return None
    s0, s1, a0, a1 = src(sub, 0), src(sub, 1), src(add, 0), src(add, 1)
    if None in (s0, s1, a0, a1):
        return None
    # subtract: x0*cos - x1*sin; add: x0*sin + x1*cos (in either operand order)
    if not (s0[0] == 0 and s1[0] == 1):
        return None
    cos_k, sin_k = s0[1], s1[1]
    if {(a0[0], a0[1]), (a1[0], a1[1])} != {(0, sin_k), (1, cos_k)} or cos_k == sin_k:
        return None
    cons = gi.consumers.get(("o", sub.id), [])
    if len(cons) != 1 or cons[0].op_name != "concatenate":
        return None
    cat = cons[0]
    if len(cat.operands) != 2 or tkey(cat.operands[0]) != ("o", sub.id) or tkey(cat.operands[1]) != ("o", add.id):
        return None
    if int(cat.attributes.get("dimension", -1)) != 3:
        return None
    cos_t, sin_t = s0[2], s1[2]
    ops += [sub, add, cat]
    if not _exclusive(gi, ops, cat):
        return None
    return cat, ops, cos_t, sin_t


def match_rope_gemm(gi: GraphIndex, dot) -> Optional[Claim]:
    """x @ Wqkv split into q, k, v heads with the half-split rotary embedding on q
    and k (qwen3_embedding/kernels/attention.py + rope.py): the rotation becomes
    the GEMM's epilogue and the rotated heads stay in place in its output."""
    if dot.op_name != "dot" or str(np.dtype(dot.result_dtype)) != "bfloat16" or len(dot.result_shape) != 3:
        return None
    if ("o", dot.id) in gi.results:
        return None
    B, S, N = (int(x) for x in dot.result_shape)
    ranges, interior, aliases, tables = [], [], {}, None
    for sl in gi.consumers.get(("o", dot.id), []):
        rng = _last_axis_slice(sl, 3)
        if rng is None:
            return None  # every use of the product must be a column slice
        users = gi.consumers.get(("o", sl.id), [])
        if len(users) != 1 or users[0].op_name != "reshape" or ("o", sl.id) in gi.results:
            continue
        rs = users[0]
        shp = tuple(int(x) for x in rs.result_shape)
        if len(shp) != 4 or shp[:2] != (B, S) or shp[2] * shp[3] != rng[1] - rng[0]:
            continue
        rot = _rotation_of(gi, rs)
        if rot is None:
            continue
        cat, ops, cos_t, sin_t = rot
        hd = shp[3]
        if tables is not None and (tkey(cos_t), tkey(sin_t), tables[2]) != (tkey(tables[0]), tkey(tables[1]), hd):
            continue
        if tuple(int(x) for x in cos_t.shape) != (S, hd // 2) or tuple(int(x) for x in sin_t.shape) != (S, hd // 2):
            continue
        if rng[0] % hd or hd not in (64, 128):
            continue
        tables = (cos_t, sin_t, hd)
        ranges.append(rng)
        interior += ops
        aliases[cat.id] = rs
    if not ranges or len(ranges) > 2:
        return None
    return Claim("rope_gemm", dot, interior, {"dot": dot, "ranges": ranges, "hd": tables[2], "cos": tables[0],
                                                 "sin": tables[1], "aliases": aliases, "seq": S})


# rmsnorm before residual_gemm: a residual add that feeds an RMSNorm belongs to the fused norm kernel
MATCHERS = (
    match_attention, match_linear_attention, match_swiglu_gemm, match_softmax, match_rmsnorm, match_argmax,
    match_residual_gemm, match_rope_gemm,
)


def find_claims(graph) -> Dict[int, Claim]:
    gi = GraphIndex(graph)
    claims: Dict[int, Claim] = {}
    taken = set()
    for op in reversed(graph.operations):
        if id(op) in taken:
            continue
        for m in MATCHERS:
            c = m(gi, op)
            if c is None:
                continue
            ids = {id(o) for o in c.interior} | {id(c.root)}
            if ids & taken:
                continue
            taken |= ids
            claims[c.root.id] = c
            break
    absorb_rope_gathers(gi, claims, taken)
    return claims, taken
