"""Lower a traced graph onto the libnkb kernel library: the fusion/tiling pass.

This is the B200 replacement for the reference's compile step
(``core/compile.py:115-309``: HLO proto -> neuronx-cc -> NEFF).  One pass
over the nodes in trace order:

* nodes claimed by a recogniser (``patterns.py``) become one fused launch
  (``softmax_rows``, ``rmsnorm_rows``, ``argmax_rows``);
* view nodes (``reshape``/``transpose``/``slice``/``broadcast``/``copy``)
  only rewrite a strided view or a lazy expression -- no launch;
* elementwise nodes extend a lazy expression; the expression is compiled
  into a single ``ew`` launch where its value is needed in memory (a
  non-elementwise consumer, a graph output, a multi-use intermediate);
* ``dot`` becomes ``gemm_bf16`` (tcgen05) when both operands are bf16 and
  TMA can describe them, ``gemm_simt`` otherwise; ``reduce`` -> ``reduce``;
  ``gather`` -> ``take`` / ``gather_pts``; ``concatenate`` writes each part
  straight into its slice of the result; ``pad``, ``dynamic-update-slice``,
  ``scatter``, ``all-reduce`` map to their kernels.

Intermediates live in one scratch arena whose offsets are packed by
lifetime.  A graph output that is a whole intermediate buffer is produced in
place in the caller's output buffer.  Anything without a lowering raises
``NotImplementedError`` at plan time: there is no host fallback.
"""

from typing import Dict, List, Optional, Union

import ml_dtypes
import numpy as np

from nkipy_b200.planner import ewprog as E
from nkipy_b200.planner import views as V
from nkipy_b200.planner.patterns import find_claims, tkey
from nkipy_b200.planner.plan import BufDecl, IoSpec, Plan, StepRec, pack_arena, pack_symmetric

Value = Union[V.View, E.Expr]

BF16 = np.dtype(ml_dtypes.bfloat16)


def _nbytes(shape, dtype) -> int:
    n = int(np.prod(shape, dtype=np.int64)) if len(shape) else 1
    return n * np.dtype(dtype).itemsize


def linattn_segments(heads, T):
    """Segments per (batch, head) of the linear-attention kernel: one, unless the
    heads alone cannot fill the GPU (fewer than 96) and the sequence is longer
    than one segment of 8 blocks of 128 tokens.  Mirrors the kernel's rule."""
    blocks = -(-T // 128)
    if blocks <= 8 or heads >= 96:
        return 1
    return -(-blocks // 8)


class Lowering:
    def __init__(self, graph, world: int = 1):
        self.g = graph
        self.world = world
        self.buffers: List[BufDecl] = []
        self.steps: List[StepRec] = []
        self.consts: List[np.ndarray] = []
        self.vals: Dict[tuple, Value] = {}
        self.uses: Dict[tuple, int] = {}
        for op in graph.operations:
            for t in op.operands:
                self.uses[tkey(t)] = self.uses.get(tkey(t), 0) + 1
        for r in graph.results:
            self.uses[tkey(r)] = self.uses.get(tkey(r), 0) + 1
        self.consumers: Dict[tuple, list] = {}
        for op in graph.operations:
            for t in op.operands:
                self.consumers.setdefault(tkey(t), []).append(op)
        self.claims, self.claimed = find_claims(graph)
        self.fused = set()  # ids of ops already lowered as part of an earlier step
        self.alias_ops: Dict[int, object] = {}  # op id -> op whose value it takes (rotated in place)
        self.needs_comm = False
        self.pos = {op.id: i for i, op in enumerate(graph.operations)}
        self.cur = -1  # position of the op being lowered
        self.mutated_params = {a.param_index for a in graph.aliases}
        self.updatable = set()  # tmp buffers written by a scatter / update-slice chain
        self.tuples: Dict[int, tuple] = {}  # op id -> views of a tuple-valued node

    # ------------------------------------------------------------ buffers
    def new_buf(self, kind, index, nbytes) -> int:
        self.buffers.append(BufDecl(kind, index, int(nbytes)))
        return len(self.buffers) - 1

    def tmp_view(self, shape, dtype) -> V.View:
        b = self.new_buf("tmp", -1, max(1, _nbytes(shape, dtype)))
        return V.View(b, 0, tuple(shape), V.dense_strides(shape), np.dtype(dtype))

    def const_view(self, arr: np.ndarray) -> V.View:
        arr = np.ascontiguousarray(arr)
        self.consts.append(arr)
        b = self.new_buf("const", len(self.consts) - 1, max(1, arr.nbytes))
        return V.View(b, 0, tuple(arr.shape), V.dense_strides(arr.shape), arr.dtype)

    def step(self, kernel, bufs, ints=(), floats=(), note=""):
        self.steps.append(StepRec(kernel, list(bufs), [int(i) for i in ints], [float(f) for f in floats], note))

    @staticmethod
    def bref(v: V.View):
        return (v.buf, v.offset * np.dtype(v.dtype).itemsize)

    # ------------------------------------------------------------ values
    def expr_of(self, val: Value) -> E.Expr:
        return val if isinstance(val, E.Expr) else E.leaf(val)

    def materialize(self, val: Value, dense=True, out: Optional[V.View] = None) -> V.View:
        """A view holding ``val``; written into ``out`` when given."""
        if isinstance(val, V.View) and out is None:
            if not dense or val.is_dense():
                return val
        if out is None:
            out = self.tmp_view(val.shape, val.dtype)
        self.emit_ew(self.expr_of(val), out)
        return out

    # ------------------------------------------------------------ in-place updates
    def _whole(self, v) -> bool:
        return (
            isinstance(v, V.View) and v.offset == 0 and v.is_dense()
            and self.buffers[v.buf].nbytes == max(1, _nbytes(v.shape, v.dtype))
        )

    def _refs_buf(self, val, b) -> bool:
        if isinstance(val, V.View):
            return val.buf == b
        return any(l.view.buf == b for l in val.leaves())

    def _pending(self, key) -> bool:
        """Is the value under ``key`` still read by an op after the current one?"""
        if key in self.result_keys:
            return True
        return any(self.pos[c.id] > self.cur for c in self.consumers.get(key, ()))

    def mutable_base(self, t, op) -> V.View:
        """A whole dense buffer holding the value of ``t`` that ``op`` (a scatter or
        dynamic-update-slice) may overwrite.

        The reference traces ``a[i] = v`` with a tensor ``i`` as ``copy(a)`` and a
        scatter (``core/ops/indexing.py:359-433``), and ``a[0:n] = v`` as a
        dynamic-update-slice of ``a`` itself (``indexing.py:692-760``,
        ``core/tensor.py:627-815``).  With ``t`` (or the tensor it copies):

        * an update result read by nothing else: the update runs in place in that
          buffer (successive ``a[...] = v`` cost no copies);
        * a parameter that the kernel mutates (its output is
          bound to the ``<name>.must_alias_input`` input): a ``copy_bytes`` step,
          which does nothing when the caller binds the same device memory to both
          (the reference's KV-cache decode, ``examples/models/qwen3/qwen3.py:289-301``).
          Values still to be read that depend on the parameter's old contents
          are materialised first, since the update may overwrite them;
        * otherwise: a copy into a new buffer.
        """
        prev = t
        src = t.source_op
        if src is not None and src.op_name == "copy" and self.uses.get(tkey(t), 0) == 1 and tkey(t) not in self.result_keys:
            prev = src.operands[0]
        pv = self.get(prev)
        sole = self.uses.get(tkey(prev), 0) == 1 and tkey(prev) not in self.result_keys
        if self._whole(pv) and self.buffers[pv.buf].kind == "tmp" and pv.buf in self.updatable and sole:
            return pv.with_(shape=tuple(op.result_shape), strides=V.dense_strides(op.result_shape))
        if self._whole(pv) and self.buffers[pv.buf].kind == "in" and self.buffers[pv.buf].index in self.mutated_params:
            b = pv.buf
            for key, val in list(self.vals.items()):
                if self._refs_buf(val, b) and self._pending(key):
                    self.vals[key] = self.materialize(val, out=self.tmp_view(val.shape, val.dtype))
            out = self.tmp_view(op.result_shape, op.result_dtype)
            self.step("copy_bytes", [self.bref(pv), self.bref(out)], [max(1, _nbytes(t.shape, t.dtype))],
                      note="mutated parameter (no-op when bound in place)")
            self.updatable.add(out.buf)
            return out
        out = self.tmp_view(op.result_shape, op.result_dtype)
        self.emit_ew(self.expr_of(self.get(t)), out)
        self.updatable.add(out.buf)
        return out

    def copy_view(self, src: V.View, dst: V.View):
        """dst = src for two strided views of one shape; views of more axes than
        the ``ew`` kernel takes (after merging) are copied in slices along
        their shortest axis."""
        try:
            self.emit_ew(E.leaf(src), dst)
            return
        except E.TooBig:
            pass
        axes = [d for d in range(len(src.shape)) if src.shape[d] > 1]
        if not axes:
            raise NotImplementedError("copy of a view the elementwise kernel cannot take")
        d = min(axes, key=lambda i: src.shape[i])
        keep = [i for i in range(len(src.shape)) if i != d]
        for i in range(int(src.shape[d])):
            self.copy_view(
                src.with_(offset=src.offset + i * src.strides[d], shape=tuple(src.shape[k] for k in keep),
                          strides=tuple(src.strides[k] for k in keep)),
                dst.with_(offset=dst.offset + i * dst.strides[d], shape=tuple(dst.shape[k] for k in keep),
                          strides=tuple(dst.strides[k] for k in keep)),
            )

    def try_transpose(self, src: V.View, dst: V.View) -> bool:
        """dst = src as one ``transpose_tiles`` launch (TMA-staged tile
        transpose) when the copy moves the innermost axis: after merging the
        axes contiguous in both views, the source's unit-stride axis C is not
        the destination's unit-stride axis R, at most three other axes remain,
        nothing is broadcast, and every stride and base offset is a multiple of
        16 bytes (the TMA rules).  Element sizes 2 and 4."""
        esize = np.dtype(src.dtype).itemsize
        if esize not in (2, 4) or np.dtype(src.dtype) != np.dtype(dst.dtype) or src.shape != dst.shape:
            return False
        if (src.offset * esize) % 16 or (dst.offset * esize) % 16 or src.size < 1024:
            return False
        shape, (ds, ss) = V.collapse(src.shape, [dst.strides, src.strides])
        if len(shape) < 2 or len(shape) > 5 or 0 in ss or 0 in ds:
            return False
        r_ax = len(shape) - 1
        if ds[r_ax] != 1 or ss[r_ax] == 1 or 1 not in ss:
            return False
        c_ax = ss.index(1)
        batch = [i for i in range(len(shape)) if i not in (c_ax, r_ax)]
        strides = [ss[r_ax], ds[c_ax]] + [s for i in batch for s in (ss[i], ds[i])]
        if any((s * esize) % 16 for s in strides):
            return False
        ints = [esize, int(shape[c_ax]), int(shape[r_ax]), int(ss[r_ax]), int(ds[c_ax]), len(batch)]
        for i in batch:
            ints += [int(shape[i]), int(ss[i]), int(ds[i])]
        self.step("transpose_tiles", [self.bref(src), self.bref(dst)], ints,
                  note=f"{tuple(src.shape)} {np.dtype(src.dtype).name} axes C={c_ax} R={r_ax}")
        return True

    def emit_ew(self, expr: E.Expr, out: V.View, depth=0):
        if expr.kind == "leaf" and self.try_transpose(expr.view, out):
            return
        try:
            c = E.compile_ew(expr, out)
        except E.TooBig:
            if depth > 16 or expr.kind != "op":
                raise
            # split: materialise the operand subtrees, then retry the root
            args = []
            for a in expr.args:
                if a.kind == "op":
                    args.append(E.leaf(self.materialize(a)))
                else:
                    args.append(a)
            root = E.Expr("op", expr.shape, expr.dtype, op=expr.op, attrs=expr.attrs, args=args)
            return self.emit_ew(root, out, depth + 1)
        bufs = [(out.buf, 0)] + [(v.buf, 0) for v in c.in_views]
        self.step("ew", bufs, c.ints, note=f"{c.n_instr} instr {tuple(out.shape)} {np.dtype(out.dtype).name}")

    def get(self, t) -> Value:
        return self.vals[tkey(t)]

    def put(self, t_or_op, val: Value):
        key = ("o", t_or_op.id)
        if isinstance(val, E.Expr) and val.kind == "op" and self.uses.get(key, 0) > 1 and key not in self.result_keys:
            # a shared intermediate is computed once
            val = self.materialize(val)
        self.vals[key] = val

    # ------------------------------------------------------------ main pass
    def run(self, name="kernel") -> Plan:
        g = self.g
        self.result_keys = {tkey(r) for r in g.results}
        inputs = []
        for p in g.parameters:
            spec = IoSpec(p.name, tuple(p.shape), np.dtype(p.dtype))
            inputs.append(spec)
            b = self.new_buf("in", p.parameter_id, max(1, spec.nbytes))
            self.vals[("p", p.parameter_id)] = V.View(b, 0, tuple(p.shape), V.dense_strides(p.shape), np.dtype(p.dtype))
        for op in g.operations:
            self.cur = self.pos[op.id]
            if op.id in self.fused:
                continue
            if op.id in self.alias_ops:
                self.vals[("o", op.id)] = self.vals[("o", self.alias_ops[op.id].id)]
                continue
            if id(op) in self.claimed and op.id not in self.claims:
                continue
            if op.id in self.claims:
                self.lower_claim(self.claims[op.id])
                continue
            fn = getattr(self, "op_" + op.op_name.replace("-", "_"), None)
            if fn is None:
                if op.op_name in E.ELEMENTWISE:
                    self.op_elementwise(op)
                    continue
                raise NotImplementedError(f"no B200 lowering for HLO op '{op.op_name}'")
            fn(op)
        outputs = []
        for i, r in enumerate(g.results):
            odt = np.dtype(np.uint8) if np.dtype(r.dtype) == np.bool_ else np.dtype(r.dtype)
            spec = IoSpec(r.name, tuple(r.shape), odt)
            outputs.append(spec)
            self.bind_output(i, r, spec)
        self.split_k()
        self.merge_launches()
        lifetimes = self.lifetimes()
        scratch = pack_arena(self.buffers, lifetimes)
        symm = pack_symmetric(self.buffers)
        aliases = [(a.output_index, a.param_index) for a in g.aliases]
        return Plan(name, inputs, outputs, self.consts, self.buffers, self.steps, scratch, aliases, self.needs_comm,
                    symm)

    def bind_output(self, i, r, spec):
        val = self.vals[tkey(r)]
        out_dt = np.dtype(np.bool_) if np.dtype(r.dtype) == np.bool_ else spec.dtype
        if isinstance(val, V.View) and val.is_dense() and val.offset == 0:
            b = self.buffers[val.buf]
            if b.kind == "tmp" and b.nbytes == max(1, spec.nbytes) and not getattr(b, "_bound", False):
                b.kind, b.index = "out", i
                b._bound = True
                return
        ob = self.new_buf("out", i, max(1, spec.nbytes))
        out_view = V.View(ob, 0, tuple(r.shape), V.dense_strides(r.shape), out_dt)
        if isinstance(val, V.View) and val.is_dense() and np.dtype(val.dtype) == out_dt and spec.nbytes > 0:
            # a dense result held elsewhere (the symmetric region of a fused all-reduce)
            self.step("copy_bytes", [self.bref(val), self.bref(out_view)], [spec.nbytes], note="result copy")
            return
        self.emit_ew(self.expr_of(val), out_view)

    # B200: 148 SMs, tcgen05 GEMM tiles of 128 x 256 x 64
    SMS, TILE_M, TILE_N, TILE_K = 148, 128, 256, 64

    def split_k(self):
        """Plain bf16 GEMMs with too few output tiles to occupy the SMs (the
        decode projections: 8 rows against a weight matrix) split their K range
        so about one work unit per SM streams its share of the weights; the
        fp32 partials go to a workspace and are summed once.  Runs after every
        fusion (an all-reduce merges only into a plain GEMM)."""
        for s in self.steps:
            if s.kernel != "gemm_bf16" or len(s.ints) != 13 or len(s.bufs) != 3:
                continue
            M, N, K = s.ints[:3]
            if s.ints[6] != 1 or s.ints[10] != 0 or M <= 0 or N <= 0:
                continue
            if self._skinny(s):
                continue
            tiles = -(-M // self.TILE_M) * -(-N // self.TILE_N)
            k_blocks = -(-K // self.TILE_K)
            if 2 * tiles > self.SMS or k_blocks < 4:
                continue
            ks = min(k_blocks // 2, self.SMS // tiles)
            if ks < 2 or ks * M * N * 4 > (256 << 20):
                continue
            ws = self.new_buf("tmp", -1, ks * M * N * 4)
            s.bufs.append((ws, 0))
            s.ints += [4, ks]
            s.note += f" split-k {ks}"

    # kernel -> (buffer refs per row set, output ref index within a set, ints per set)
    _MERGEABLE = {"rmsnorm_rope_rows": (6, 2, 12), "scatter_rows": (3, 0, 6)}

    def merge_launches(self):
        """Two adjacent launches of the same row kernel, neither of which reads or
        writes what the other writes, run as one launch over both row sets (the
        decode step's q and k RMSNorm + rotary, and its K and V cache-row
        scatters): one launch gap less each."""
        def disjoint(x, y):
            return not ({i for i, _ in x.bufs} & {i for i, _ in y.bufs})

        merged = []
        for s in self.steps:
            spec = self._MERGEABLE.get(s.kernel)
            if spec and merged and merged[-1].kernel != s.kernel:
                # an earlier launch of the same kernel behind at most two steps that
                # touch none of its buffers (the copy of a mutated cache into its
                # output): those steps move ahead of it, so that the two meet
                for back in (2, 3):
                    if len(merged) >= back and merged[-back].kernel == s.kernel and all(
                            disjoint(merged[-back], m) for m in merged[-back + 1:]):
                        merged.append(merged.pop(-back))
                        break
            prev = merged[-1] if merged else None
            if prev is not None and spec and prev.kernel == s.kernel and self._independent(prev, s, spec):
                nb, _, ni = spec
                a, b = list(prev.ints), list(s.ints)
                if s.kernel == "scatter_rows":  # both sets carry upd_pre_bytes
                    a = a if len(a) == 6 else a + [a[4] * a[3]]
                    b = b if len(b) == 6 else b + [b[4] * b[3]]
                if (len(prev.bufs) == nb and len(s.bufs) == nb and len(a) == ni and len(b) == ni
                        and prev.floats == s.floats
                        and (s.kernel != "rmsnorm_rope_rows" or (a[1], a[2]) == (b[1], b[2]))):
                    prev.bufs = prev.bufs + s.bufs
                    prev.ints = a + b
                    prev.note = f"{prev.note} | {s.note}"
                    continue
            merged.append(s)
        self.steps = merged

    def _independent(self, a, b, spec) -> bool:
        """Neither launch touches the other's output buffer (by buffer, not range)."""
        _, oi, _ = spec
        if len(a.bufs) != spec[0] or len(b.bufs) != spec[0]:
            return False
        out_a, out_b = a.bufs[oi][0], b.bufs[oi][0]
        return out_a not in {x for x, _ in b.bufs} and out_b not in {x for x, _ in a.bufs}

    def _skinny(self, s) -> bool:
        """At most 16 rows of A (K contiguous) against B (N contiguous): the
        ``gemm_skinny`` kernel (mma.sync with the rows as one m16 tile, B
        streamed once), its K range split for two CTAs per SM."""
        M, N, K, lda, ldb, ldc = s.ints[:6]
        a_mn, b_k = s.ints[11], s.ints[12]
        if M > 16 or a_mn or b_k or K % 8 or N % 8 or lda % 8 or ldb % 8 or ldc % 2:
            return False
        if s.bufs[0][1] % 16 or s.bufs[1][1] % 16 or s.bufs[2][1] % 4:
            return False
        col_blocks = -(-N // 256)
        splits = max(1, 2 * self.SMS // col_blocks)  # at most one wave of two CTAs per SM
        kc = min(1024, max(64, -(-(-(-K // splits)) // 64) * 64))
        ks = -(-K // kc)
        ws = self.new_buf("tmp", -1, ks * M * N * 4 if ks > 1 else 16)
        # B that no step writes (a constant, or an input not updated in place)
        # may be read while the previous kernel drains
        bb = self.buffers[s.bufs[1][0]]
        b_pre = int(bb.kind == "const" or (bb.kind == "in" and bb.index not in self.mutated_params))
        s.kernel = "gemm_skinny"
        s.bufs = s.bufs[:3] + [(ws, 0)]
        s.ints = [M, N, K, lda, ldb, ldc, kc, b_pre]
        s.note = f"{M}x{N}x{K} k-ranges {ks}"
        return True

    def lifetimes(self):
        life = {}
        for si, s in enumerate(self.steps):
            for bid, _ in s.bufs:
                lo, hi = life.get(bid, (si, si))
                life[bid] = (min(lo, si), max(hi, si))
        return life

    # ------------------------------------------------------------ claims
    def dense_rows(self, t):
        v = self.materialize(self.get(t), dense=True)
        cols = int(t.shape[-1]) if t.shape else 1
        rows = int(np.prod(t.shape[:-1])) if len(t.shape) > 1 else 1
        return v, rows, cols

    def row_blocks(self, t):
        """``(view, rows, cols, block_rows, block_stride)`` for a row kernel's
        input: its rows read in place when they come in equally spaced blocks
        of dense rows (per-head rows of a fused projection's output), else a
        dense copy (one block)."""
        val = self.get(t)
        cols = int(t.shape[-1]) if t.shape else 1
        rows = int(np.prod(t.shape[:-1])) if len(t.shape) > 1 else 1
        if isinstance(val, V.View) and not val.is_dense() and rows > 0 and cols > 0:
            shp, (st,) = V.collapse(val.shape, [val.strides])
            if len(shp) == 2 and st[1] == 1 and shp[1] % cols == 0 and st[0] >= shp[1]:
                return val, rows, cols, shp[1] // cols, int(st[0])
        v, rows, cols = self.dense_rows(t)
        return v, rows, cols, rows, rows * cols

    def lower_rmsnorm_rope(self, p, wv, out, shape):
        """Per-head RMSNorm with the rotary embedding in its epilogue: one
        ``rmsnorm_rope_rows`` launch reading the cos / sin rows itself (at the
        run-time position for a gathered row, per token for a prefill table)."""
        rp = p["rope"]
        half = shape[3] // 2
        tshape = (int(rp["rows"]), half)
        tabs = []
        for t in (rp["cos"], rp["sin"]):
            v = self.get(t)
            st = V.reshape_strides(v.shape, v.strides, tshape) if isinstance(v, V.View) else None
            if st is None or st[1] != 1:
                v = self.materialize(v, dense=True)
                st = V.dense_strides(tshape)
            tabs.append(v.with_(shape=tshape, strides=tuple(int(x) for x in st)))
        cv, sv = tabs
        if tshape[0] > 1 and cv.strides[0] != sv.strides[0]:
            cv, sv = (self.materialize(v, dense=True) for v in tabs)
        ts = int(cv.strides[0]) if tshape[0] > 1 else half
        xv, rows, cols, blk, bstride = self.row_blocks(p["x"])
        if rp["pos"] is not None:
            posv = self.materialize(self.get(rp["pos"]), dense=True)
            has_pos, pos_dt = 1, E.dt_code(posv.dtype)
        else:
            posv, has_pos, pos_dt = cv, 0, 0
        B, S, H, _ = shape
        ints = [rows, cols, E.dt_code(wv.dtype), blk, bstride, ts, has_pos, pos_dt, int(cv.shape[0]), S, H,
                rp["per_token"]]
        self.step(
            "rmsnorm_rope_rows",
            [self.bref(xv), self.bref(wv), self.bref(out), self.bref(cv), self.bref(sv), self.bref(posv)],
            ints,
            [p["eps"]],
            note=f"{rows}x{cols} + rotary ({'position' if has_pos else 'per token' if rp['per_token'] else 'row 0'})",
        )

    def lower_claim(self, c):
        root = c.root
        if c.kind == "softmax":
            x = c.params["x"]
            xv, rows, cols = self.dense_rows(x)
            if np.dtype(xv.dtype) not in (np.dtype(np.float32), BF16):
                raise NotImplementedError("softmax on this dtype")
            out = self.tmp_view(root.result_shape, c.params["out_dtype"])
            self.step(
                "softmax_rows",
                [self.bref(xv), self.bref(out)],
                [rows, cols, E.dt_code(xv.dtype), E.dt_code(out.dtype)],
                note=f"{rows}x{cols}",
            )
            self.vals[("o", root.id)] = out
        elif c.kind == "rmsnorm":
            p = c.params
            out = self.tmp_view(root.result_shape, p["out_dtype"])
            wv = self.materialize(self.get(p["w"]), dense=True)
            dt = np.dtype(p["out_dtype"])
            if p["residual"] is not None:
                a, b = p["residual"]
                av, rows, cols = self.dense_rows(a)
                bv, _, _ = self.dense_rows(b)
                hs = self.tmp_view(p["sum_tensor"].shape, p["sum_tensor"].dtype) if p["sum_needed"] else None
                bufs = [self.bref(av), self.bref(bv), self.bref(wv), self.bref(out), self.bref(hs if hs else out)]
                self.step(
                    "rmsnorm_rows",
                    bufs,
                    [rows, cols, E.dt_code(dt), E.dt_code(wv.dtype), 1, 1 if hs else 0],
                    [p["eps"]],
                    note=f"{rows}x{cols} residual{'+sum' if hs else ''}",
                )
                if hs is not None:
                    self.vals[tkey(p["sum_tensor"])] = hs
            elif p.get("rope") is not None:
                self.lower_rmsnorm_rope(p, wv, out, tuple(int(d) for d in root.result_shape))
            else:
                xv, rows, cols, blk, bstride = self.row_blocks(p["x"])
                bufs = [self.bref(xv), self.bref(xv), self.bref(wv), self.bref(out), self.bref(out)]
                ints = [rows, cols, E.dt_code(dt), E.dt_code(wv.dtype), 0, 0]
                if blk != rows:
                    ints += [blk, bstride]
                self.step(
                    "rmsnorm_rows",
                    bufs,
                    ints,
                    [p["eps"]],
                    note=f"{rows}x{cols}" + (f" in blocks of {blk} rows, stride {bstride}" if blk != rows else ""),
                )
            self.vals[("o", root.id)] = out
        elif c.kind == "attention":
            self.lower_attention(c)
        elif c.kind == "swiglu_gemm":
            self.lower_swiglu(c)
        elif c.kind == "residual_gemm":
            self.lower_residual_gemm(c)
        elif c.kind == "rope_gemm":
            self.lower_rope_gemm(c)
        elif c.kind == "linattn":
            self.lower_linattn(c)
        elif c.kind == "argmax":
            x = c.params["x"]
            xv, rows, cols = self.dense_rows(x)
            out = self.tmp_view(root.result_shape, np.int32)
            self.step(
                "argmax_rows",
                [self.bref(xv), self.bref(out)],
                [rows, cols, E.dt_code(xv.dtype), 1 if c.params["is_max"] else 0],
                note=f"{rows}x{cols}",
            )
            self.vals[("o", root.id)] = out
        else:
            raise NotImplementedError(c.kind)

    def lower_attention(self, c):
        p = c.params
        root = c.root

        def strided(t, amap, heads_div=1):
            v = self.get(t)
            if not isinstance(v, V.View) or v.strides[amap[3]] != 1:
                v = self.materialize(v, dense=True)
            st = v.strides
            return v, [st[amap[0]], st[amap[1]], st[amap[2]], st[amap[3]]]

        qv, qs = strided(p["q"], p["q_map"])
        kv, ks = strided(p["k"], p["k_map"])
        vv, vs = strided(p["v"], p["v_map"])
        B, H, S, D = p["batch"], p["heads"], p["sq"], p["d"]
        k_heads = int(p["k"].shape[p["k_map"][1]])
        if p["n_rep"] == 1 and k_heads != H:
            raise NotImplementedError("attention with mismatched head counts")
        # output stored (B, S, H, D): the traced transpose(0,2,1,3) after it is free
        out = self.tmp_view((B, S, H, D), BF16)
        if p.get("pos") is not None:
            # one query row against keys 0..pos of the cache: split over keys, then merged
            posv = self.materialize(self.get(p["pos"]), dense=True)
            skv = p["skv"]
            # chunks of ~512 keys (eight 16-key tiles per warp, double-buffered), at
            # least one CTA per SM in all, at most 256 chunks of 16 or more keys
            bg = max(1, B * k_heads)
            splits = max(1, min(256, -(-skv // 16), max(-(-skv // 512), -(-148 // bg))))
            ws = self.tmp_view((B * H * splits * (D + 2),), np.float32)
            ints = [B, H, k_heads, skv, D, splits, E.dt_code(posv.dtype)]
            ints += qs[:2] + ks[:3] + vs[:3] + [H * D, D]
            self.step(
                "attn_decode",
                [self.bref(qv), self.bref(kv), self.bref(vv), self.bref(out), self.bref(posv), self.bref(ws)],
                ints,
                [p["scale"]],
                note=f"decode B{B} H{H}/{k_heads} L{skv} D{D} x{splits}",
            )
            self.vals[("o", root.id)] = out.with_(shape=(B, H, S, D), strides=(S * H * D, D, H * D, 1))
            return
        ints = [B, H, k_heads, S, p.get("kv_len", p["skv"]), D, int(p["causal"])]
        ints += qs[:3] + ks[:3] + vs[:3] + [S * H * D, D, H * D]
        self.step(
            "flash_attn",
            [self.bref(qv), self.bref(kv), self.bref(vv), self.bref(out)],
            ints,
            [p["scale"]],
            note=f"B{B} H{H}/{k_heads} S{S} D{D} causal={int(p['causal'])}",
        )
        self.vals[("o", root.id)] = out.with_(shape=(B, H, S, D), strides=(S * H * D, D, H * D, 1))

    def lower_linattn(self, c):
        p = c.params
        B, H, T, D = p["shape"]
        views = []
        for t in (p["q"], p["k"], p["v"]):
            v = self.get(t)
            if not isinstance(v, V.View) or v.strides[3] != 1 or any(st % 8 for st in v.strides[:3]):
                v = self.materialize(v, dense=True)
            views.append(v)
        out = self.tmp_view((B, H, T, D), BF16)
        G = linattn_segments(B * H, T)
        ws = self.new_buf("tmp", -1, max(1, B * H * G * (D * D + D) * 4) if G > 1 else 256)
        ints = [B, H, T, D, G]
        for v in views:
            ints += list(v.strides[:3])
        ints += list(out.strides[:3])
        self.step(
            "linattn",
            [self.bref(views[0]), self.bref(views[1]), self.bref(views[2]), self.bref(out), (ws, 0)],
            ints,
            note=f"B{B} H{H} T{T} D{D} segments={G}",
        )
        self.vals[("o", c.root.id)] = out

    def lower_rope_gemm(self, c):
        """q, k, v = split(x @ Wqkv) with the rotary embedding of q and k in the
        GEMM epilogue: the rotated heads stay in place in the product, and each
        traced concatenate of rotated halves takes the view of its heads."""
        if self.op_dot(c.params["dot"], epilogue=("rope", c, c.root)):
            for cat_id, rs in c.params["aliases"].items():
                self.alias_ops[cat_id] = rs
            return
        # the plain product was emitted: the rotations lower op by op where they stand
        self.claimed -= {id(o) for o in c.interior}

    def lower_residual_gemm(self, c):
        """x @ W + R with the add in the GEMM epilogue; the generic path otherwise."""
        root = c.root
        if self.op_dot(c.params["dot"], epilogue=("add", c.params["res"], root)):
            return
        a, b = (self.expr_of(self.get(t)) for t in root.operands)
        self.put(root, E.op("add", [a, b], tuple(root.result_shape), np.dtype(root.result_dtype)))

    def lower_swiglu(self, c):
        """gate/up GEMM with silu(gate) * up in the epilogue; generic path otherwise."""
        d = c.params["dot"]
        F = c.params["n_half"]
        root = c.root
        ok = self.op_dot(d, epilogue=("swiglu", F, root))
        if ok:
            return
        # fallback: the dot result exists in full; evaluate the activation as one ew group
        full = self.expr_of(self.get(d))
        n = len(d.result_shape)

        def half(i):
            starts = [0] * (n - 1) + [i * F]
            limits = list(d.result_shape[:-1]) + [(i + 1) * F]
            return E.t_slice(full, starts, limits, [1] * n)

        g, u = half(0), half(1)
        shape, bf = tuple(root.result_shape), BF16
        one = E.const(1.0, bf, shape)
        t = E.op("negate", [g], shape, bf)
        t = E.op("exponential", [t], shape, bf)
        t = E.op("add", [one, t], shape, bf)
        t = E.op("divide", [one, t], shape, bf)
        t = E.op("multiply", [g, t], shape, bf)
        self.vals[("o", root.id)] = E.op("multiply", [t, u], shape, bf)

    # ------------------------------------------------------------ view ops
    def op_reshape(self, op):
        v = self.get(op.operands[0])
        shape = tuple(op.result_shape)
        if isinstance(v, V.View):
            st = V.reshape_strides(v.shape, v.strides, shape)
            if st is None:
                v = self.materialize(v)
                st = V.dense_strides(shape)
            self.put(op, v.with_(shape=shape, strides=st))
            return
        e = E.t_reshape(v, shape)
        if e is None:
            m = self.materialize(v)
            self.put(op, m.with_(shape=shape, strides=V.dense_strides(shape)))
        else:
            self.put(op, e)

    def op_broadcast(self, op):
        v = self.get(op.operands[0])
        shape = tuple(op.result_shape)
        bd = list(op.attributes.get("broadcast_dimensions", []))
        if isinstance(v, V.View):
            self.put(op, v.with_(shape=shape, strides=V.broadcast_strides(v.shape, v.strides, shape, bd)))
        else:
            self.put(op, E.t_broadcast(v, shape, bd))

    def op_transpose(self, op):
        v = self.get(op.operands[0])
        perm = list(op.attributes["permutation"])
        if isinstance(v, V.View):
            self.put(
                op, v.with_(shape=tuple(v.shape[p] for p in perm), strides=V.transpose_strides(v.strides, perm))
            )
        else:
            self.put(op, E.t_transpose(v, perm))

    def op_slice(self, op):
        v = self.get(op.operands[0])
        a = op.attributes
        starts, limits, steps = a["start_indices"], a["limit_indices"], a["strides"]
        if isinstance(v, V.View):
            off, st = V.slice_view(v.offset, v.strides, starts, steps)
            self.put(op, v.with_(offset=off, shape=tuple(op.result_shape), strides=st))
        else:
            self.put(op, E.t_slice(v, starts, limits, steps))

    def op_copy(self, op):
        self.put(op, self.get(op.operands[0]))

    def op_constant(self, op):
        val = op.attributes.get("value")
        if isinstance(val, np.ndarray) and val.ndim > 0:
            arr = np.asarray(val).astype(op.result_dtype)
            if np.dtype(op.result_dtype) == np.bool_:
                arr = arr.astype(np.uint8)
                v = self.const_view(arr).with_(dtype=np.dtype(np.bool_))
            else:
                v = self.const_view(arr)
            self.vals[("o", op.id)] = v
            return
        if isinstance(val, np.ndarray):
            val = val.item()
        self.vals[("o", op.id)] = E.const(val, op.result_dtype, op.result_shape)

    def op_iota(self, op):
        self.vals[("o", op.id)] = E.iota(op.result_shape, op.result_dtype, op.attributes["iota_dimension"])

    # ------------------------------------------------------------ elementwise
    def op_elementwise(self, op):
        args = [self.expr_of(self.get(t)) for t in op.operands]
        e = E.op(op.op_name, args, op.result_shape, op.result_dtype, op.attributes)
        if e.n_nodes() > 48 or len(e.leaves()) > 6:
            args = [E.leaf(self.materialize(a)) if a.kind == "op" else a for a in args]
            e = E.op(op.op_name, args, op.result_shape, op.result_dtype, op.attributes)
        self.put(op, e)

    def op_convert(self, op):
        src = op.operands[0]
        if np.dtype(src.dtype) == np.dtype(op.result_dtype):
            self.put(op, self.get(src))
        else:
            self.op_elementwise(op)

    # ------------------------------------------------------------ reduce
    def op_reduce(self, op):
        x = op.operands[0]
        xv = self.materialize(self.get(x), dense=False)
        init_op = op.operands[1].source_op
        init = float(np.asarray(init_op.attributes["value"]).reshape(()).item()) if init_op is not None else 0.0
        comp = {"add": 0, "maximum": 1, "minimum": 2, "multiply": 3}[op.attributes["computation"]]
        dims = sorted(op.attributes["dimensions"])
        outer = [d for d in range(len(x.shape)) if d not in dims]
        out = self.tmp_view(op.result_shape, op.result_dtype)

        def grouped(axes):
            if not axes:
                return (), ()
            shp, (st,) = V.collapse([xv.shape[d] for d in axes], [tuple(xv.strides[d] for d in axes)])
            if shp == (1,) and all(xv.shape[d] == 1 for d in axes):
                return (1,), (0,)
            return shp, st

        oshape, ostr = grouped(outer)
        ishape, istr = grouped(dims)
        if len(oshape) > 4 or len(ishape) > 4:
            xv = self.materialize(xv, dense=True)
            oshape, ostr = grouped(outer)
            ishape, istr = grouped(dims)
        n_outer = int(np.prod(oshape)) if oshape else 1
        n_inner = int(np.prod(ishape)) if ishape else 1
        ints = [E.dt_code(xv.dtype), E.dt_code(out.dtype), comp, len(oshape), len(ishape), xv.offset, n_outer, n_inner]
        ints += list(oshape) + list(ostr) + list(ishape) + list(istr)
        self.step("reduce", [(xv.buf, 0), self.bref(out)], ints, [init], note=f"{n_outer}x{n_inner}")
        self.vals[("o", op.id)] = out

    # ------------------------------------------------------------ dot
    def op_dot(self, op, epilogue=None):
        a_t, b_t = op.operands
        at = op.attributes
        lb, rb = list(at["lhs_batch_dimensions"]), list(at["rhs_batch_dimensions"])
        lc, rc = list(at["lhs_contracting_dimensions"]), list(at["rhs_contracting_dimensions"])
        av = self.materialize(self.get(a_t), dense=False)
        bv = self.materialize(self.get(b_t), dense=False)
        na, nb = len(a_t.shape), len(b_t.shape)
        if len(lc) != 1 or len(rc) != 1:
            raise NotImplementedError("dot with several contracting dimensions")
        a_free = [d for d in range(na) if d not in lb and d not in lc]
        b_free = [d for d in range(nb) if d not in rb and d not in rc]
        if lb != list(range(len(lb))) or rb != list(range(len(rb))) or len(a_free) > 1 or len(b_free) > 1:
            raise NotImplementedError("dot layout outside the matmul form")
        M = int(a_t.shape[a_free[0]]) if a_free else 1
        N = int(b_t.shape[b_free[0]]) if b_free else 1
        K = int(a_t.shape[lc[0]])
        a_ms = av.strides[a_free[0]] if a_free else 0
        a_ks = av.strides[lc[0]]
        b_ks = bv.strides[rc[0]]
        b_ns = bv.strides[b_free[0]] if b_free else 0
        bshape = [int(a_t.shape[d]) for d in lb]
        a_bst = [av.strides[d] for d in lb]
        b_bst = [bv.strides[d] for d in rb]
        out_dt = np.dtype(op.result_dtype)
        if epilogue is not None:
            out = self.tmp_view(epilogue[2].result_shape, out_dt)
        else:
            out = self.tmp_view(op.result_shape, out_dt)
        # fold a broadcast rhs (weights shared across the batch) into M
        if bshape and all(s == 0 for s in b_bst) and M > 0:
            shp, (st,) = V.collapse(bshape + [M], [tuple(a_bst + [a_ms])])
            if len(shp) == 1:
                bshape, a_bst, b_bst, M, a_ms = [], [], [], int(shp[0]), st[0]
        batch = int(np.prod(bshape)) if bshape else 1
        # collapse the batch axes of A, B and C together
        c_bst = list(V.dense_strides(tuple(bshape) + (M, N)))[: len(bshape)] if bshape else []
        if len(bshape) > 1:
            shp, sts = V.collapse(bshape, [tuple(a_bst), tuple(b_bst), tuple(c_bst)])
            if len(shp) > 1:
                if epilogue is not None:
                    self.op_dot(op)
                    return False
                av = self.materialize(av, dense=True)
                bv = self.materialize(bv, dense=True)
                return self.op_dot_dense(op, av, bv, out)
            a_bst, b_bst, c_bst = [sts[0][0]], [sts[1][0]], [sts[2][0]]
        sA = a_bst[0] if a_bst else 0
        sB = b_bst[0] if b_bst else 0
        sC = c_bst[0] if c_bst else 0
        if M == 1 and not a_free:
            a_ms = K
        if N == 1 and not b_free:
            b_ns = 1
        is_bf = np.dtype(av.dtype) == BF16 and np.dtype(bv.dtype) == BF16 and out_dt in (BF16, np.dtype(np.float32))
        a_mn = a_ms == 1 and a_ks != 1
        a_k = a_ks == 1
        b_n = b_ns == 1
        b_k = b_ks == 1 and b_ns != 1
        eb = np.dtype(BF16).itemsize

        def aligned(v, *strides):
            return (v.offset * eb) % 16 == 0 and all(int(s) % 8 == 0 for s in strides)

        use_tc = (
            is_bf
            and K > 0
            and (a_k or a_mn)
            and (b_n or b_k)
            and (batch == 1 or (sA != 0 and sB != 0))
            and aligned(av, a_ks if a_mn else a_ms, sA)
            and aligned(bv, b_ks if b_n else b_ns, sB)
        )
        if epilogue is not None and epilogue[0] == "rope":
            cl = epilogue[1]
            cosv = self.materialize(self.get(cl.params["cos"]), dense=True)
            sinv = self.materialize(self.get(cl.params["sin"]), dense=True)
            ok = (use_tc and out_dt == BF16 and batch == 1 and N % 8 == 0
                  and all(np.dtype(v.dtype) == BF16 and (v.offset * eb) % 16 == 0 for v in (cosv, sinv)))
            if not ok:
                self.op_dot(op)
                return False
            rngs = list(cl.params["ranges"]) + [(0, 0)] * (2 - len(cl.params["ranges"]))
            lda = a_ms if a_k else a_ks
            ldb = b_ks if b_n else b_ns
            self.step(
                "gemm_bf16",
                [self.bref(av), self.bref(bv), self.bref(out), self.bref(cosv), self.bref(sinv)],
                [M, N, K, lda, ldb, N, 1, 0, 0, 0, 0, int(a_mn and not a_k), int(b_k and not b_n), 3,
                 cl.params["hd"], cl.params["seq"], rngs[0][0], rngs[0][1], rngs[1][0], rngs[1][1]],
                note=f"tc {M}x{N}x{K} +rope",
            )
            self.vals[("o", op.id)] = out
            return True
        if epilogue is not None and epilogue[0] == "add":
            rv = self.materialize(self.get(epilogue[1]), dense=True)
            if not (use_tc and out_dt == BF16 and batch == 1 and (rv.offset * eb) % 16 == 0 and N % 8 == 0):
                self.op_dot(op)
                return False
            lda = a_ms if a_k else a_ks
            ldb = b_ks if b_n else b_ns
            self.step(
                "gemm_bf16",
                [self.bref(av), self.bref(bv), self.bref(out), self.bref(rv)],
                [M, N, K, lda, ldb, N, 1, 0, 0, 0, 0, int(a_mn and not a_k), int(b_k and not b_n), 2, N],
                note=f"tc {M}x{N}x{K} +residual",
            )
            self.vals[("o", epilogue[2].id)] = out
            return True
        if epilogue is not None:
            F = epilogue[1]
            if not (use_tc and b_n and out_dt == BF16 and F % 64 == 0 and N == 2 * F and batch == 1):
                self.op_dot(op)
                return False
            lda = a_ms if a_k else a_ks
            self.step(
                "gemm_bf16",
                [self.bref(av), self.bref(bv), self.bref(out)],
                [M, F, K, lda, b_ks, F, 1, 0, 0, 0, 0, int(a_mn and not a_k), 0, 1, F],
                note=f"tc {M}x{F}(x2)x{K} +swiglu",
            )
            self.vals[("o", epilogue[2].id)] = out
            return True
        if use_tc:
            lda = a_ms if a_k else a_ks
            ldb = b_ks if b_n else b_ns
            self.step(
                "gemm_bf16",
                [self.bref(av), self.bref(bv), self.bref(out)],
                [M, N, K, lda, ldb, N, batch, sA, sB, sC, int(out_dt == np.float32), int(a_mn and not a_k), int(b_k and not b_n)],
                note=f"tc {batch}x{M}x{N}x{K}",
            )
        else:
            self.step(
                "gemm_simt",
                [self.bref(av), self.bref(bv), self.bref(out)],
                [E.dt_code(av.dtype), E.dt_code(bv.dtype), E.dt_code(out_dt), M, N, K, batch, a_ms, a_ks, b_ks, b_ns, N, 1, sA, sB, sC],
                note=f"simt {batch}x{M}x{N}x{K}",
            )
        self.vals[("o", op.id)] = out

    def op_dot_dense(self, op, av, bv, out):
        """Matmul-form dot with dense operands (batch axes flattened)."""
        a_t, b_t = op.operands
        M, K = int(a_t.shape[-2]), int(a_t.shape[-1])
        N = int(b_t.shape[-1])
        batch = int(np.prod(a_t.shape[:-2]))
        out_dt = np.dtype(op.result_dtype)
        is_bf = np.dtype(av.dtype) == BF16 and np.dtype(bv.dtype) == BF16 and out_dt in (BF16, np.dtype(np.float32))
        if is_bf and K % 8 == 0 and N % 8 == 0 and K > 0:
            self.step(
                "gemm_bf16",
                [self.bref(av), self.bref(bv), self.bref(out)],
                [M, N, K, K, N, N, batch, M * K, K * N, M * N, int(out_dt == np.float32), 0, 0],
                note=f"tc {batch}x{M}x{N}x{K}",
            )
        else:
            self.step(
                "gemm_simt",
                [self.bref(av), self.bref(bv), self.bref(out)],
                [E.dt_code(av.dtype), E.dt_code(bv.dtype), E.dt_code(out_dt), M, N, K, batch, K, 1, N, 1, N, 1, M * K, K * N, M * N],
                note=f"simt {batch}x{M}x{N}x{K}",
            )
        self.vals[("o", op.id)] = out

    # ------------------------------------------------------------ data movement
    def op_concatenate(self, op):
        dim = op.attributes["dimension"]
        out = self.tmp_view(op.result_shape, op.result_dtype)
        pos = 0
        for t in op.operands:
            n = int(t.shape[dim])
            starts = [0] * len(op.result_shape)
            starts[dim] = pos
            off, st = V.slice_view(out.offset, out.strides, starts, [1] * len(starts))
            part = out.with_(offset=off, shape=tuple(t.shape), strides=st)
            self.emit_ew(self.expr_of(self.get(t)), part)
            pos += n
        self.vals[("o", op.id)] = out

    def op_pad(self, op):
        x = op.operands[0]
        xv = self.materialize(self.get(x), dense=True)
        cfg = op.attributes["padding_config"]
        if any(c[2] != 0 or c[0] < 0 or c[1] < 0 for c in cfg):
            raise NotImplementedError("pad with interior or negative padding")
        pv = op.operands[1].source_op.attributes["value"]
        bits = int.from_bytes(np.asarray(pv, dtype=op.result_dtype).reshape(1).tobytes(), "little")
        out = self.tmp_view(op.result_shape, op.result_dtype)
        r = len(x.shape)
        ints = [r, np.dtype(op.result_dtype).itemsize, out.size, bits]
        ints += list(x.shape) + list(op.result_shape) + [c[0] for c in cfg]
        self.step("pad", [self.bref(xv), self.bref(out)], ints)
        self.vals[("o", op.id)] = out

    def op_convolution(self, op):
        """``conv2d`` / ``conv3d`` (``core/ops/conv.py:230-312``) as one GEMM.

        One ``im2col`` launch writes the window matrix, ordered (channel, kernel
        offset) x (batch, output position), from the dense input with zeros
        where a window reaches into the padding (its writes contiguous along the
        innermost output axis; other element sizes take a ``pad`` launch and a
        strided ``ew`` copy of the same matrix).  The correlation
        is then cols^T^T @ W^T: the window matrix is an M-major left operand
        (C*prod(k) rows of B*P positions) and the weight, row-major
        (OC, C, *k), a K-major right operand as it lies; with a multiple of 8
        output positions per image (bf16) it is instead one batched product
        per image, out[b] = W @ cols[:, b], the weight shared by the images
        and the result written in the (B, OC, *out) layout directly.  Otherwise
        the (B, P, OC) product is moved to the (B, OC, *out) result layout.  bf16 runs on
        ``gemm_bf16`` (fp32 accumulation), other dtypes on ``gemm_simt``.
        """
        x, w = op.operands
        a = op.attributes
        n = len(x.shape) - 2
        sp = list(range(2, 2 + n))
        std = (
            a.get("input_batch_dimension", 0) == 0 and a.get("input_feature_dimension", 1) == 1
            and list(a.get("input_spatial_dimensions", sp)) == sp
            and a.get("kernel_output_feature_dimension", 0) == 0 and a.get("kernel_input_feature_dimension", 1) == 1
            and list(a.get("kernel_spatial_dimensions", sp)) == sp
            and a.get("output_batch_dimension", 0) == 0 and a.get("output_feature_dimension", 1) == 1
            and list(a.get("output_spatial_dimensions", sp)) == sp
        )
        if not std or a.get("feature_group_count", 1) != 1 or a.get("batch_group_count", 1) != 1:
            raise NotImplementedError("convolution outside NC-spatial layout with one feature group")
        if any(int(d) != 1 for d in a.get("lhs_dilation", [1] * n)):
            raise NotImplementedError("convolution with input dilation")
        stride = [int(s) for s in a["window_strides"]]
        pads = [(int(lo), int(hi)) for lo, hi in a["padding"]]
        dil = [int(d) for d in a.get("rhs_dilation", [1] * n)]
        B, C = int(x.shape[0]), int(x.shape[1])
        OC, ks = int(w.shape[0]), tuple(int(k) for k in w.shape[2:])
        out_sp = tuple(int(s) for s in op.result_shape[2:])
        dt = np.dtype(op.result_dtype)
        xv = self.materialize(self.get(x), dense=True)
        P, KK = int(np.prod(out_sp)), C * int(np.prod(ks))
        M, N, K = B * P, OC, KK
        cols = self.tmp_view((KK, M), x.dtype)  # cols[kk, b * P + p], zero where a window reaches the padding
        es = np.dtype(x.dtype).itemsize
        if es in (2, 4):
            ints = [n, es, B, C] + [int(d) for d in x.shape[2:]] + list(ks) + list(out_sp) + stride
            ints += [lo for lo, _ in pads] + dil
            self.step("im2col", [self.bref(xv), self.bref(cols)], ints, note="convolution windows")
        else:
            if any(lo or hi for lo, hi in pads):
                pshape = (B, C) + tuple(int(x.shape[2 + i]) + pads[i][0] + pads[i][1] for i in range(n))
                pv = self.tmp_view(pshape, x.dtype)
                ints = [n + 2, es, pv.size, 0] + [int(s_) for s_ in x.shape] + list(pshape)
                ints += [0, 0] + [lo for lo, _ in pads]
                self.step("pad", [self.bref(xv), self.bref(pv)], ints, note="convolution padding")
                xv = pv
            xs = xv.strides
            win = xv.with_(
                shape=(C,) + ks + (B,) + out_sp,
                strides=(xs[1],) + tuple(xs[2 + i] * dil[i] for i in range(n)) + (xs[0],)
                + tuple(xs[2 + i] * stride[i] for i in range(n)),
            )
            self.copy_view(win, cols.with_(shape=win.shape, strides=V.dense_strides(win.shape)))
        wv = self.materialize(self.get(w), dense=True)
        eb = np.dtype(BF16).itemsize
        bf = np.dtype(cols.dtype) == BF16 and np.dtype(wv.dtype) == BF16 and dt == BF16
        if bf and K % 8 == 0 and P % 8 == 0 and M % 8 == 0 and (wv.offset * eb) % 16 == 0:
            # per image: out[b] (OC x P) = W (OC x K, shared by every image) @ cols[:, b] (K x P),
            # written straight in the (B, OC, *out) result layout
            out = self.tmp_view((B, OC) + out_sp, dt)
            self.step("gemm_bf16", [self.bref(wv), self.bref(cols), self.bref(out)],
                      [OC, P, K, K, M, P, B, 0, P, OC * P, 0, 0, 0], note=f"tc {B}x{OC}x{P}x{K} convolution")
            self.put(op, out)
            return
        prod = self.tmp_view((B, P, OC), dt)
        if (np.dtype(cols.dtype) == BF16 and np.dtype(wv.dtype) == BF16 and dt == BF16 and K % 8 == 0
                and N % 8 == 0 and M % 8 == 0 and (wv.offset * eb) % 16 == 0):
            self.step("gemm_bf16", [self.bref(cols), self.bref(wv), self.bref(prod)],
                      [M, N, K, M, K, N, 1, 0, 0, 0, 0, 1, 1], note=f"tc {M}x{N}x{K} convolution")
        else:
            self.step("gemm_simt", [self.bref(cols), self.bref(wv), self.bref(prod)],
                      [E.dt_code(cols.dtype), E.dt_code(wv.dtype), E.dt_code(dt), M, N, K, 1, 1, M, 1, K, N, 1, 0, 0, 0],
                      note=f"simt {M}x{N}x{K} convolution")
        # (B, P, OC) -> (B, OC, *out)
        moved = prod.with_(shape=(B, OC) + out_sp,
                           strides=(P * OC, 1) + tuple(s * OC for s in V.dense_strides(out_sp)))
        self.put(op, moved)

    def op_dynamic_update_slice(self, op):
        base, upd = op.operands[0], op.operands[1]
        starts = []
        for t in op.operands[2:]:
            sop = t.source_op
            if sop is None or sop.op_name != "constant":
                raise NotImplementedError("dynamic-update-slice with run-time start indices")
            starts.append(int(np.asarray(sop.attributes["value"]).reshape(()).item()))
        out = self.mutable_base(base, op)
        starts = [max(0, min(s, int(n) - int(u))) for s, n, u in zip(starts, base.shape, upd.shape)]
        off, st = V.slice_view(out.offset, out.strides, starts, [1] * len(starts))
        self.emit_ew(self.expr_of(self.get(upd)), out.with_(offset=off, shape=tuple(upd.shape), strides=st))
        self.vals[("o", op.id)] = out

    def op_gather(self, op):
        x, ind = op.operands
        a = op.attributes
        xv = self.materialize(self.get(x), dense=True)
        iv = self.materialize(self.get(ind), dense=True)
        out = self.tmp_view(op.result_shape, op.result_dtype)
        r = len(x.shape)
        es = np.dtype(op.result_dtype).itemsize
        cs = list(a["collapsed_slice_dims"])
        if len(cs) == 1 and list(a["start_index_map"]) == cs and a["index_vector_dim"] == len(ind.shape):
            ax = cs[0]
            pre = int(np.prod(x.shape[:ax])) if ax else 1
            post = int(np.prod(x.shape[ax + 1 :])) if ax + 1 < r else 1
            n_idx = int(np.prod(ind.shape)) if len(ind.shape) else 1
            self.step(
                "take",
                [self.bref(xv), self.bref(iv), self.bref(out)],
                [E.dt_code(iv.dtype), pre, int(x.shape[ax]), post * es, n_idx],
                note=f"take axis {ax}",
            )
        elif not a["offset_dims"] and cs == list(range(r)) and a["index_vector_dim"] == len(ind.shape) - 1:
            n = int(np.prod(op.result_shape)) if len(op.result_shape) else 1
            ints = [E.dt_code(iv.dtype), r, es, n] + [int(s) for s in x.shape] + list(V.dense_strides(x.shape))
            self.step("gather_pts", [self.bref(xv), self.bref(iv), self.bref(out)], ints, note="point gather")
        else:
            raise NotImplementedError("gather form outside take / take_along_axis")
        self.vals[("o", op.id)] = out

    def op_scatter(self, op):
        x, ind, upd = op.operands
        a = op.attributes
        if a.get("update_computation", "assign") != "assign":
            raise NotImplementedError("scatter with a combiner")
        iv = self.materialize(self.get(ind), dense=True)
        ue = self.get(upd)
        if np.dtype(upd.dtype) != np.dtype(op.result_dtype):
            # NumPy casts the assigned values to the array's dtype; the kernels copy bytes
            ue = E.op("convert", [self.expr_of(ue)], tuple(upd.shape), np.dtype(op.result_dtype))
        upd_blocks = None  # (block elements, block stride) of an update view read in place
        if isinstance(ue, V.View) and not ue.is_dense():
            shp, (st,) = V.collapse(ue.shape, [ue.strides])
            if len(shp) == 2 and st[1] == 1 and st[0] >= shp[1]:
                upd_blocks = (int(shp[0]), int(shp[1]), int(st[0]))
        uv = ue if upd_blocks else self.materialize(ue, dense=True)
        r = len(x.shape)
        es = np.dtype(op.result_dtype).itemsize
        ins = list(a["inserted_window_dims"])
        xs, us = tuple(int(d) for d in x.shape), tuple(int(d) for d in upd.shape)
        if (len(ins) == 1 and len(us) == r - 1 and int(np.prod(ind.shape)) == 1
                and list(a["update_window_dims"]) == [d for d in range(r) if d != ins[0]]):
            # one index and an update without the indexed axis (``x[i] = row`` with a
            # one-element index array): the window form with that axis of size 1
            us = us[: ins[0]] + (1,) + us[ins[0]:]
        window = (
            len(ins) == 1
            and list(a["update_window_dims"]) == [d for d in range(r) if d != ins[0]]
            and len(us) == r
            and len(ind.shape) <= 1
            and us[: ins[0]] == xs[: ins[0]]
            and us[ins[0] + 1 :] == xs[ins[0] + 1 :]
        )
        points = not a["update_window_dims"] and ins == list(range(r))
        if not (window or points):
            raise NotImplementedError("scatter form")
        out = self.mutable_base(x, op)
        if window:
            # whole windows along one axis: updates are (pre, n_idx, post), dense
            ax = ins[0]
            pre = int(np.prod(x.shape[:ax])) if ax else 1
            post = int(np.prod(x.shape[ax + 1 :])) if ax + 1 < r else 1
            n_idx = int(np.prod(ind.shape)) if len(ind.shape) else 1
            ints = [E.dt_code(iv.dtype), pre, int(x.shape[ax]), post * es, n_idx]
            if upd_blocks:
                nb, blk, bst = upd_blocks
                if nb == pre and blk == n_idx * post:
                    ints.append(bst * es)  # (n_idx, post) dense per pre block: read in place
                else:
                    uv = self.materialize(uv, dense=True)
            self.step("scatter_rows", [self.bref(out), self.bref(iv), self.bref(uv)], ints)
        else:
            if upd_blocks:
                uv = self.materialize(uv, dense=True)
            n = int(np.prod(upd.shape)) if len(upd.shape) else 1
            ints = [E.dt_code(iv.dtype), r, es, n] + [int(s) for s in x.shape] + list(V.dense_strides(x.shape))
            self.step("scatter_pts", [self.bref(out), self.bref(iv), self.bref(uv)], ints)
        self.vals[("o", op.id)] = out

    def op_topk(self, op):
        """Last-axis top-k (``core/ops/nn.py:65-152``): one ``topk_rows`` launch
        writing the values and the uint32 indices; the two ``get-tuple-element``
        nodes that follow take them."""
        x = op.operands[0]
        k = int(op.attributes["k"])
        if not op.attributes.get("largest", True):
            raise NotImplementedError("topk with largest = false")
        xv, rows, cols = self.dense_rows(x)
        shape = tuple(op.result_shape)
        vals = self.tmp_view(shape, x.dtype)
        idx = self.tmp_view(shape, np.uint32)
        bufs = [self.bref(xv), self.bref(vals), self.bref(idx)]
        ints = [rows, cols, k, E.dt_code(xv.dtype)]
        if k <= 32 and rows > 0:
            # room for the one-pass kernel's per-part key lists: up to 64 parts of
            # k rounded up to 8, 16 or 32 keys per row
            kl = 8 if k <= 8 else 16 if k <= 16 else 32
            keys = rows * min(64, max(1, cols // 4096)) * kl
            ws = self.new_buf("tmp", -1, keys * 8)
            bufs.append((ws, 0))
            ints.append(keys)
        self.step("topk_rows", bufs, ints, note=f"{rows}x{cols} k={k}")
        self.tuples[op.id] = (vals, idx)

    def op_get_tuple_element(self, op):
        src = op.operands[0].source_op
        if src is None or src.id not in self.tuples:
            raise NotImplementedError("get-tuple-element of a node without a tuple lowering")
        self.vals[("o", op.id)] = self.tuples[src.id][int(op.attributes["tuple_index"])]

    def _gather_dim(self, op, key):
        groups = op.attributes.get("replica_groups") or [[0]]
        if len(groups) != 1 or len(groups[0]) != self.world:
            raise ValueError(
                f"{op.op_name} over groups {groups} but the kernel is planned for world size {self.world}"
            )
        return int(op.attributes[key]) % max(1, len(op.operands[0].shape))

    def op_all_gather(self, op):
        """Concatenation of every rank's tensor along ``all_gather_dim``
        (``core/ops/collectives.py:34-53``): NCCL gathers rank-major into a
        (world, *shape) buffer; the concatenation is a view of it (a move to
        the gather axis when it is not the leading one)."""
        x = op.operands[0]
        d = self._gather_dim(op, "all_gather_dim")
        if self.world == 1:
            self.put(op, self.get(x))
            return
        xv = self.materialize(self.get(x), dense=True)
        shp = tuple(int(s) for s in x.shape)
        g = self.tmp_view((self.world,) + shp, x.dtype)
        self.needs_comm = True
        self.step("allgather", [self.bref(xv), self.bref(g)], [xv.size, E.dt_code(xv.dtype)],
                  note=f"{xv.size} x {self.world}")
        self._concat_ranks(op, g, d)

    def _rank_blocks(self, x, d):
        """``x`` split into world blocks along axis ``d``, laid out rank-major as
        a dense (world, *block) buffer (a view when ``d`` is the leading axis)."""
        shp = tuple(int(s) for s in x.shape)
        if shp[d] % self.world:
            raise ValueError(f"axis {d} of {shp} does not split over {self.world} ranks")
        blk = shp[:d] + (shp[d] // self.world,) + shp[d + 1:]
        src = self.get(x)
        if d == 0:
            return self.materialize(src, dense=True), blk
        split = shp[:d] + (self.world, shp[d] // self.world) + shp[d + 1:]
        perm = [d] + [i for i in range(len(split)) if i != d]
        e = E.t_reshape(self.expr_of(src), split)
        if e is None:
            m = self.materialize(src)
            e = E.leaf(m.with_(shape=split, strides=V.dense_strides(split)))
        sv = self.tmp_view((self.world,) + blk, x.dtype)
        self.emit_ew(E.t_transpose(e, perm), sv)
        return sv, blk

    def _concat_ranks(self, op, g, d):
        """Bind a (world, *block) buffer as the concatenation of its blocks along ``d``."""
        n = len(g.shape) - 1
        perm = list(range(1, d + 1)) + [0] + list(range(d + 1, n + 1))
        moved = g.with_(shape=tuple(g.shape[p] for p in perm), strides=V.transpose_strides(g.strides, perm))
        self.op_reshape_value(op, moved)

    def op_reduce_scatter(self, op):
        """Sum over the ranks, each keeping its block of ``reduce_scatter_dim``
        (``core/ops/collectives.py:148-178``): the blocks laid out rank-major,
        then one NCCL reduce-scatter."""
        x = op.operands[0]
        if op.attributes.get("reduce_op", "add") not in ("add", np.add):
            raise NotImplementedError("reduce-scatter other than sum")
        d = self._gather_dim(op, "reduce_scatter_dim")
        if self.world == 1:
            self.put(op, self.get(x))
            return
        sv, blk = self._rank_blocks(x, d)
        out = self.tmp_view(blk, x.dtype)
        self.needs_comm = True
        n = int(np.prod(blk)) if blk else 1
        self.step("reducescatter", [self.bref(sv), self.bref(out)], [n, E.dt_code(out.dtype)], note=f"{n} per rank")
        self.vals[("o", op.id)] = out

    def op_all_to_all(self, op):
        """Block j of ``split_dimension`` goes to rank j; the blocks received
        are concatenated in rank order (``core/ops/collectives.py:217-233``,
        whose traced result keeps the input shape, so the split and concat
        axes must agree)."""
        x = op.operands[0]
        a = op.attributes
        d = self._gather_dim(op, "split_dimension")
        if int(a["concat_dimension"]) % max(1, len(x.shape)) != d:
            raise NotImplementedError("all-to-all with different split and concat axes")
        if self.world == 1:
            self.put(op, self.get(x))
            return
        sv, blk = self._rank_blocks(x, d)
        g = self.tmp_view((self.world,) + blk, x.dtype)
        self.needs_comm = True
        n = int(np.prod(blk)) if blk else 1
        self.step("alltoall", [self.bref(sv), self.bref(g)], [n, E.dt_code(g.dtype)], note=f"{n} per block")
        self._concat_ranks(op, g, d)

    def op_reshape_value(self, op, v):
        """Bind ``v`` reshaped to ``op``'s result shape (a view when possible)."""
        shape = tuple(op.result_shape)
        st = V.reshape_strides(v.shape, v.strides, shape)
        if st is None:
            v = self.materialize(v)
            st = V.dense_strides(shape)
        self.put(op, v.with_(shape=shape, strides=st))

    def op_all_reduce(self, op):
        """Sum over the ranks, in place in symmetric memory.

        The partial sum is produced straight into a "symm" buffer (one region
        that every rank maps, bound to the communicator when the plan is
        loaded), where the runtime reduces it inside NVSwitch, or with NCCL
        when no such region is bound.  An add of the reduced value to one
        other tensor of its shape (the residual after a row-parallel block) is
        folded into the same step.
        """
        x = op.operands[0]
        if op.attributes.get("reduce_op", "add") != "add":
            raise NotImplementedError("all-reduce other than sum")
        groups = op.attributes.get("replica_groups") or [[0]]
        if len(groups[0]) != self.world:
            raise ValueError(
                f"all-reduce over {len(groups[0])} ranks but the kernel is planned for world size {self.world}"
            )
        if self.world == 1:
            self.put(op, self.get(x))
            return
        xv = self.materialize(self.get(x), dense=True)
        esize = np.dtype(xv.dtype).itemsize
        b = self.buffers[xv.buf]
        if (b.kind == "tmp" and xv.offset == 0 and b.nbytes == xv.size * esize
                and self.uses.get(tkey(x), 0) == 1 and tkey(x) not in self.result_keys):
            b.kind = "symm"  # the producer writes into the symmetric region
        else:
            sb = self.new_buf("symm", -1, max(1, xv.size * esize))
            sv = V.View(sb, 0, tuple(op.result_shape), V.dense_strides(op.result_shape), np.dtype(xv.dtype))
            self.emit_ew(self.expr_of(xv), sv)
            xv = sv
        dt = E.dt_code(xv.dtype)
        self.needs_comm = True
        add = self._residual_add(op)
        gemm = self._fusable_gemm(xv)
        if gemm is not None:
            # the GEMM that produced the partial sum reduces it itself, tile
            # row block by row block, as its tiles are stored
            gemm.kernel = "gemm_bf16_ar"
            gemm.ints.append(0)  # flag slot (launches of the plan are ordered, so they share one)
            gemm.note += " +all-reduce"
            if add is not None:
                add_op, other = add
                rv = self.materialize(self.get(other), dense=True)
                gemm.bufs.append(self.bref(rv))
                gemm.note += " +residual"
                self.vals[("o", add_op.id)] = xv
                self.fused.add(add_op.id)
                return
            self.vals[("o", op.id)] = xv
            return
        if add is not None:
            add_op, other = add
            rv = self.materialize(self.get(other), dense=True)
            out = self.tmp_view(add_op.result_shape, add_op.result_dtype)
            self.step("allreduce_add", [self.bref(xv), self.bref(rv), self.bref(out)], [xv.size, dt],
                      note=f"{xv.size} + residual")
            self.vals[("o", add_op.id)] = out
            self.fused.add(add_op.id)
            return
        self.step("allreduce", [self.bref(xv), self.bref(xv)], [xv.size, dt], note=f"{xv.size} in place")
        self.vals[("o", op.id)] = xv

    def _fusable_gemm(self, xv):
        """The step that just wrote ``xv`` when it is a plain bf16 GEMM whose
        dense output is exactly ``xv`` (one batch, no epilogue); else None."""
        if not self.steps:
            return None
        s = self.steps[-1]
        if s.kernel != "gemm_bf16" or len(s.ints) != 13 or len(s.bufs) != 3:
            return None
        M, N, _K, _lda, _ldb, ldc, batch = s.ints[:7]
        if s.bufs[2] != self.bref(xv) or s.ints[10] != 0 or batch != 1 or ldc != N or N % 8:
            return None
        if np.dtype(xv.dtype).itemsize != 2 or xv.size != M * N:
            return None
        return s

    def _residual_add(self, op):
        """(add op, other operand) when the all-reduce result's only use is an
        unclaimed add with a same-shape, same-dtype tensor; else None."""
        key = ("o", op.id)
        users = self.consumers.get(key, [])
        if self.uses.get(key, 0) != 1 or len(users) != 1 or key in self.result_keys:
            return None
        u = users[0]
        if u.op_name != "add" or len(u.operands) != 2:
            return None
        rms = self._rmsnorm_of_residual(u)
        if (id(u) in self.claimed or u.id in self.claims) and rms is None:
            return None
        a, c = u.operands
        other = c if tkey(a) == key else a
        if tkey(other) == key or tuple(other.shape) != tuple(op.result_shape):
            return None
        if np.dtype(other.dtype) != np.dtype(op.result_dtype) or np.dtype(u.result_dtype) != np.dtype(op.result_dtype):
            return None
        if np.dtype(op.result_dtype) not in (np.dtype(np.float32), BF16):
            return None
        if rms is not None:
            # the residual + RMSNorm recogniser claimed this add: the all-reduce
            # applies it, and the norm reads the sum (one read and one write of
            # the activations less)
            rms.params["residual"] = None
            rms.params["x"] = rms.params["sum_tensor"]
        return u, other

    def _rmsnorm_of_residual(self, add_op):
        """The residual + RMSNorm claim whose residual sum is ``add_op``, or None."""
        for c in self.claims.values():
            if c.kind == "rmsnorm" and c.params.get("residual") is not None:
                st = c.params.get("sum_tensor")
                if st is not None and st.source_op is add_op:
                    return c
        return None


def lower(graph, name=None, world: int = 1) -> Plan:
    return Lowering(graph, world=world).run(name or graph.name)
