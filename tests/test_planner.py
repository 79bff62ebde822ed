"""Planner unit tests (CPU): view algebra, fusion decisions, plan format."""

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200 import workloads as W
from nkipy_b200.core import ops as cc_ops
from nkipy_b200.core.ops import collectives as cc
from nkipy_b200.core.trace import NKIPyKernel
from nkipy_b200.planner import ewprog as E
from nkipy_b200.planner import lower
from nkipy_b200.planner import views as V

BF16 = np.dtype(ml_dtypes.bfloat16)


def plan_of(fn, *args, **kw):
    return lower(NKIPyKernel.trace(fn).specialize(*args, **kw))


@pytest.mark.parametrize(
    "shape,perm_or_none,new_shape",
    [((4, 6), None, (24,)), ((4, 6), None, (2, 2, 6)), ((2, 3, 4), (1, 0, 2), (6, 4)), ((3, 4), (1, 0), (12,))],
)
def test_reshape_strides_matches_numpy(shape, perm_or_none, new_shape):
    a = np.arange(int(np.prod(shape))).reshape(shape)
    st = V.dense_strides(shape)
    if perm_or_none is not None:
        a = a.transpose(perm_or_none)
        st = V.transpose_strides(st, perm_or_none)
    got = V.reshape_strides(a.shape, st, new_shape)
    try:
        r = a.view()
        r.shape = new_shape  # numpy raises when a copy would be needed
        want = tuple(s // a.itemsize for s in r.strides)
    except AttributeError:
        want = None
    if want is None:
        assert got is None
    else:
        flat = np.arange(int(np.prod(shape))).reshape(shape)
        idx = np.indices(new_shape).reshape(len(new_shape), -1)
        offs = sum(i * s for i, s in zip(idx, got))
        np.testing.assert_array_equal(flat.reshape(-1)[offs], r.reshape(-1))


def test_collapse_merges_contiguous_axes():
    shp, sets = V.collapse((4, 5, 6), [(30, 6, 1), (0, 0, 1)])
    assert shp == (20, 6) and sets == [(6, 1), (0, 1)]


@pytest.mark.parametrize(
    "name,args,kernels",
    [
        ("softmax", W.make_inputs("softmax", scale=1 / 512), {"softmax_rows": 1}),
        ("rmsnorm", W.make_inputs("rmsnorm", scale=1 / 2048), {"rmsnorm_rows": 1}),
        ("gemm", W.make_inputs("gemm", scale=1 / 64), {"gemm_bf16": 1}),
        ("bmm", W.make_inputs("bmm", scale=1 / 32), {"gemm_bf16": 1}),
    ],
)
def test_config_kernels_plan_to_one_fused_launch(name, args, kernels):
    p = plan_of(W.KERNELS[name], *args)
    assert p.kernel_counts() == kernels


def test_elementwise_chain_is_one_launch():
    def k(x, w):
        return np.tanh(x * 2.0 + w[None, :]) - np.exp(-x)

    p = plan_of(k, np.zeros((8, 16), np.float32), np.zeros(16, np.float32))
    assert p.kernel_counts() == {"ew": 1}


def test_plan_text_roundtrip_fields():
    p = plan_of(W.softmax_kernel, np.zeros((4, 64), np.float32))
    t = p.to_text()
    assert t.startswith("NKBPLAN 1") and t.rstrip().endswith("end")
    assert "step softmax_rows" in t


def test_bool_output_is_bytes():
    p = plan_of(lambda x: x > 0, np.zeros((3, 3), np.float32))
    assert np.dtype(p.outputs[0].dtype) == np.uint8


def test_unsupported_op_fails_loudly():
    def k(x):
        return cc.all_to_all(x, split_dimension=0, concat_dimension=1, replica_groups=[[0, 1]])

    with pytest.raises(NotImplementedError):
        lower(NKIPyKernel.trace(k).specialize(np.zeros((4, 8), np.float32)), world=2)


def test_topk_is_one_launch_with_two_results():
    from nkipy_b200.core.ops import nn

    def k(x):
        v, i = nn.topk(x, 5, axis=-1)
        return v, i

    p = plan_of(k, np.zeros((4, 100), np.float32))
    assert p.kernel_counts() == {"topk_rows": 1}
    assert [np.dtype(o.dtype) for o in p.outputs] == [np.dtype(np.float32), np.dtype(np.uint32)]
    # both results are written straight into the output buffers; the fourth buffer
    # holds the one-pass kernel's per-part key lists (1 part of 8 keys per row here)
    assert [p.buffers[b].kind for b, _ in p.steps[0].bufs[1:]] == ["out", "out", "tmp"]
    assert p.steps[0].ints == [4, 100, 5, E.dt_code(np.float32), 4 * 8]


def _ag0(x):
    return cc.all_gather(x, all_gather_dim=0, replica_groups=[[0, 1]])


def _ag1(x):
    return cc.all_gather(x, all_gather_dim=1, replica_groups=[[0, 1]])


def _rs0(x):
    return cc.reduce_scatter(x, reduce_scatter_dim=0, replica_groups=[[0, 1]])


def _rs1(x):
    return cc.reduce_scatter(x, reduce_scatter_dim=1, replica_groups=[[0, 1]])


def _a2a1(x):
    return cc.all_to_all(x, split_dimension=1, concat_dimension=1, replica_groups=[[0, 1]])


@pytest.mark.parametrize(
    "fn,kernels",
    [
        (_ag0, ["allgather"]),  # rank-major gather is the concatenation itself
        (_ag1, ["allgather", "ew"]),  # ... moved to the gather axis
        (_rs0, ["reducescatter"]),
        (_rs1, ["ew", "reducescatter"]),  # blocks laid out rank-major first
        (_a2a1, ["ew", "alltoall", "ew"]),
    ],
)
def test_collective_plans_world2(fn, kernels):
    p = lower(NKIPyKernel.trace(fn).specialize(np.zeros((8, 16), np.float32)), world=2)
    assert [s.kernel for s in p.steps] == kernels and p.needs_comm


def _cache_decode_plan():
    B, L, nq, nkv, hd, D = 2, 64, 4, 2, 128, 512
    kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
    z = np.zeros((B, L, nkv, hd), BF16)
    args = (np.zeros((B, 1, D), BF16), np.zeros((D, (nq + 2 * nkv) * hd), BF16), np.ones(hd, BF16), np.ones(hd, BF16),
            z, z, np.array([3], np.int32), np.zeros((nq * hd, D), BF16))
    return plan_of(W.cached_attention_kernel, *args, **kw), z.nbytes


def test_kv_cache_decode_updates_caches_in_place():
    p, cache_bytes = _cache_decode_plan()
    assert sorted(p.aliases) == [(1, 4), (2, 5)]
    copies = [s for s in p.steps if s.kernel == "copy_bytes"]
    # one copy per cache, from the mutated input into its output (a no-op when bound in place)
    assert [(p.buffers[s.bufs[0][0]].kind, p.buffers[s.bufs[0][0]].index) for s in copies] == [("in", 4), ("in", 5)]
    assert [(p.buffers[s.bufs[1][0]].kind, p.buffers[s.bufs[1][0]].index) for s in copies] == [("out", 1), ("out", 2)]
    assert all(s.ints == [cache_bytes] for s in copies)
    # the new token's rows are scattered into the output buffers (both caches in one
    # launch: the copy of the V cache moves ahead of the K scatter); no other step
    # writes a whole cache
    (sc,) = [s for s in p.steps if s.kernel == "scatter_rows"]
    assert [p.buffers[sc.bufs[i][0]].kind for i in (0, 3)] == ["out", "out"]
    assert [p.buffers[sc.bufs[i][0]].index for i in (0, 3)] == [1, 2]
    cache_ins = {i for i, b in enumerate(p.buffers) if b.kind == "in" and b.index in (4, 5)}
    assert not any(s.kernel == "ew" and s.bufs[1][0] in cache_ins for s in p.steps)
    # the attention of the new token is one fused step reading the updated caches
    kinds = [s.kernel for s in p.steps]
    assert kinds.count("attn_decode") == 1
    dec = p.steps[kinds.index("attn_decode")]
    assert kinds.index("attn_decode") > max(i for i, k in enumerate(kinds) if k == "scatter_rows")
    assert {p.buffers[dec.bufs[i][0]].kind for i in (1, 2)} == {"out"}
    assert dec.ints[:7] == [2, 4, 2, 64, 128, dec.ints[5], 3] and dec.floats == [pytest.approx(128 ** -0.5)]
    # per-head q/k RMSNorm + rotary: one launch over both row sets, rows read in place
    # from the QKV projection, the cos / sin rows read at the run-time position (no
    # gather launch)
    width = (4 + 2 * 2) * 128
    (rr,) = [s for s in p.steps if s.kernel == "rmsnorm_rope_rows"]
    sets = [rr.ints[:12], rr.ints[12:]]
    assert [q[3:5] for q in sets] == [[4, width], [2, width]]
    assert all(q[6] == 1 and q[8] == 64 and q[11] == 0 for q in sets)
    assert all(p.buffers[rr.bufs[i][0]].kind == "in" and p.buffers[rr.bufs[i][0]].index == 6 for i in (5, 11))
    # the 2-row projections run on the skinny GEMM (rows as one m16 tile), K split into
    # 64-row ranges: 8 of them, each CTA's fp32 partial rows in the workspace; the
    # weights (inputs no step writes) may be read while the previous kernel drains
    gs = [s for s in p.steps if s.kernel == "gemm_skinny"]
    assert [s.ints for s in gs] == [[2, width, 512, 512, width, width, 64, 1], [2, 512, 512, 512, 512, 512, 64, 1]]
    assert [p.buffers[s.bufs[3][0]].nbytes for s in gs] == [8 * 2 * width * 4, 8 * 2 * 512 * 4]
    assert "gemm_bf16" not in kinds
    # the new value row is scattered straight from the projection output
    assert len(sc.ints) == 12 and sc.ints[11] == width * 2
    assert not {"ew", "take", "rmsnorm_rows"} & set(kinds)


def test_cache_prefill_norm_and_rotary_fused_per_token():
    B, L, nq, nkv, hd, D, S = 2, 128, 8, 2, 128, 1024, 32
    kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
    z = np.zeros((B, L, nkv, hd), BF16)
    p = plan_of(W.cached_attention_kernel, np.zeros((B, S, D), BF16), np.zeros((D, (nq + 2 * nkv) * hd), BF16),
                np.ones(hd, BF16), np.ones(hd, BF16), z, z, None, np.zeros((nq * hd, D), BF16), **kw)
    (rr,) = [s for s in p.steps if s.kernel == "rmsnorm_rope_rows"]  # q and k row sets in one launch
    # rows, cols, w dtype, block rows, block stride, table stride, has_pos, pos dtype, table rows, S, H, per token
    width = (nq + 2 * nkv) * hd
    assert rr.ints == [B * S * nq, hd, 1, nq, width, hd // 2, 0, 0, S, S, nq, 1,
                       B * S * nkv, hd, 1, nkv, width, hd // 2, 0, 0, S, S, nkv, 1]
    # the NumPy cos / sin tables (one constant node per use) are read from one constant each
    assert {p.buffers[rr.bufs[i][0]].kind for i in (3, 4, 9, 10)} == {"const"}
    assert "take" not in p.kernel_counts()
    # mask[:S, :L] is causal over the first S cache rows: one flash launch reading S keys
    # of the updated caches
    (fa,) = [s for s in p.steps if s.kernel == "flash_attn"]
    assert fa.ints[:7] == [B, nq, nkv, S, S, hd, 1]
    assert [p.buffers[fa.bufs[i][0]].kind for i in (1, 2)] == ["out", "out"]
    assert fa.ints[10:13] == [L * nkv * hd, hd, nkv * hd]


def test_readers_of_a_mutated_parameter_run_before_its_update():
    def k(a, idx, v):
        old = a * 2.0
        a[:, idx] = v
        return old + a

    a = np.zeros((6, 10, 5), np.float32)
    p = plan_of(k, a, np.array([7], np.int32), np.zeros((6, 1, 5), np.float32))
    kinds = [s.kernel for s in p.steps]
    first_write = kinds.index("copy_bytes")
    reads_a = [i for i, s in enumerate(p.steps) if any(p.buffers[b].kind == "in" and p.buffers[b].index == 0
                                                       for b, _ in s.bufs)]
    assert reads_a and all(i <= first_write for i in reads_a)


def test_successive_updates_share_one_buffer():
    def k(a, i, j, v, w):
        a[i] = v
        a[j] = w
        a[0:2] = 0.0
        return a.sum(axis=1)

    a = np.zeros((9, 33), np.float32)
    r = np.zeros((1, 33), np.float32)
    p = plan_of(k, a, np.array([4], np.int32), np.array([7], np.int32), r, r)
    assert p.kernel_counts()["copy_bytes"] == 1
    writes = {s.bufs[0][0] for s in p.steps if s.kernel in ("scatter_rows", "copy_bytes")}
    dst = {s.bufs[1][0] for s in p.steps if s.kernel == "copy_bytes"}
    assert writes - {b for b, _ in [s.bufs[0] for s in p.steps if s.kernel == "copy_bytes"]} == dst


def test_ew_program_budget_split():
    def k(x):
        y = x
        for i in range(40):
            y = np.tanh(y * 1.01 + float(i))
        return y

    p = plan_of(k, np.zeros((4, 4), np.float32))
    assert all(s.kernel == "ew" for s in p.steps)
    assert len(p.steps) >= 2


def test_ew_compile_bf16_rounding_inserted():
    x = E.leaf(V.View(0, 0, (4,), (1,), BF16))
    e = E.op("add", [x, x], (4,), BF16)
    c = E.compile_ew(e, V.View(1, 0, (4,), (1,), BF16))
    prog = c.ints[7 + 1 + 1 + 1 + (2 + 1) :]
    instrs = [prog[i : i + 8] for i in range(0, len(prog), 8)]
    add = [ins for ins in instrs if ins[0] == E.OP["FADD"]]
    assert len(add) == 1 and add[0][6] == 1  # rounded to bf16 by the add itself


def test_ew_constant_operand_is_immediate():
    x = E.leaf(V.View(0, 0, (4,), (1,), np.dtype(np.float32)))
    e = E.op("multiply", [E.const(2.0, np.float32, (4,)), x], (4,), np.float32)
    c = E.compile_ew(e, V.View(1, 0, (4,), (1,), np.dtype(np.float32)))
    assert c.n_instr == 2  # load + multiply-by-immediate


def test_layer_plans(monkeypatch):
    s = W.LayerShape(batch=1, seq=64, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512)
    full = W.layer_weights(s, seed=0)
    shard = W.shard_layer_weights(full, s, 0, 1)
    x = np.zeros((1, 64, 256), BF16)
    args, kw = W.layer_args(x, shard, s, 1)
    p = plan_of(W.llama_decoder_layer_kernel, *args, **kw)
    counts = p.kernel_counts()
    # RoPE in the QKV GEMM epilogue, SwiGLU in the gate/up epilogue, the last
    # residual add in the down projection's epilogue: no elementwise launch left
    assert counts == {"rmsnorm_rows": 2, "gemm_bf16": 4, "flash_attn": 1}
    notes = [s.note for s in p.steps if s.kernel == "gemm_bf16"]
    assert any("+rope" in n for n in notes) and any("+swiglu" in n for n in notes)
    assert any("+residual" in n for n in notes)


def test_layer_tp2_fuses_allreduces_into_gemms():
    s = W.LayerShape(batch=1, seq=64, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512)
    full = W.layer_weights(s, seed=0)
    shard = W.shard_layer_weights(full, s, 1, 2)
    args, kw = W.layer_args(np.zeros((1, 64, 256), BF16), shard, s, 2)
    p = lower(NKIPyKernel.trace(W.llama_decoder_layer_kernel).specialize(*args, **kw), world=2)
    kc = p.kernel_counts()
    assert any("+rope" in s.note for s in p.steps) and p.needs_comm
    # each row-parallel GEMM reduces its own partial sum and adds the residual after it (the
    # first one's add is also the residual of the post-attention RMSNorm, which then reads the sum)
    assert kc["gemm_bf16_ar"] == 2 and "allreduce" not in kc and "allreduce_add" not in kc
    ar = [s for s in p.steps if s.kernel == "gemm_bf16_ar"]
    assert [len(s.bufs) for s in ar] == [4, 4] and all(len(s.ints) == 14 for s in ar)
    norms = [s for s in p.steps if s.kernel == "rmsnorm_rows"]
    assert norms[1].ints[4] == 0 and norms[1].bufs[0][0] == ar[0].bufs[2][0]
    # the second all-reduce's residual is the first one's result, in the symmetric region
    assert ar[1].bufs[3][0] == ar[0].bufs[2][0]
    # both partial sums live in the symmetric region; the layer output is copied out of it
    symm = [i for i, b in enumerate(p.buffers) if b.kind == "symm"]
    assert sorted(s.bufs[2][0] for s in ar) == symm and p.symm >= sum(p.buffers[i].nbytes for i in symm)
    assert "ew" not in kc and p.steps[-1].kernel == "copy_bytes" and p.steps[-1].bufs[0][0] == ar[1].bufs[2][0]
    assert "symm %d" % p.symm in p.to_text()


def test_allreduce_without_gemm_stays_a_step():
    def k(x, r):
        return r + cc.all_reduce(x * 2.0, replica_groups=[[0, 1]], reduce_op=np.add)

    x = np.zeros((64, 256), BF16)
    p = lower(NKIPyKernel.trace(k).specialize(x, x), world=2)
    assert p.kernel_counts().get("allreduce_add") == 1 and "gemm_bf16_ar" not in p.kernel_counts()


def test_convolution_plans():
    def c2(x, w, b):
        return cc_ops.conv2d(x, w, b, stride=1, padding=1)

    def c3(x, w):
        return cc_ops.conv3d(x, w, stride=(1, 2, 1), padding=1, dilation=(2, 1, 1))

    p = plan_of(c2, np.zeros((2, 16, 12, 12), BF16), np.zeros((32, 16, 3, 3), BF16), np.zeros(32, BF16))
    # window matrix (padding as zeros), tensor-core GEMM, layout move fused with the bias add
    assert [s.kernel for s in p.steps] == ["im2col", "gemm_bf16", "ew"]
    assert p.steps[0].ints == [2, 2, 2, 16, 12, 12, 3, 3, 12, 12, 1, 1, 1, 1, 1, 1]
    p = plan_of(c3, np.zeros((1, 2, 6, 7, 8), np.float32), np.zeros((3, 2, 2, 3, 2), np.float32))
    kinds = p.kernel_counts()
    assert kinds["gemm_simt"] == 1 and kinds["im2col"] == 1 and "pad" not in kinds
    (im,) = [s for s in p.steps if s.kernel == "im2col"]
    # 3-D: input 6x7x8, kernel 2x3x2, output 6x4x9, stride (1, 2, 1), low padding 1, dilation (2, 1, 1)
    assert im.ints == [3, 4, 1, 2, 6, 7, 8, 2, 3, 2, 6, 4, 9, 1, 2, 1, 1, 1, 1, 2, 1, 1]


def test_skinny_gemm_selection():
    """At most 16 rows with K-contiguous A and N-contiguous B take the skinny
    mma.sync GEMM; more rows or a transposed operand keep the tcgen05 kernel."""
    def mm(a, b):
        return a @ b

    def mm_bt(a, b):
        return a @ b.T

    z = lambda *s: np.zeros(s, BF16)  # noqa: E731
    p = plan_of(mm, z(16, 4096), z(4096, 1024))
    (s,) = p.steps
    M, N, K, lda, ldb, ldc, kc, b_pre = s.ints
    assert s.kernel == "gemm_skinny" and (M, N, K, lda, ldb, ldc) == (16, 1024, 4096, 4096, 1024, 1024)
    assert b_pre == 1  # B is a plan input that no step writes
    # B computed by an earlier step: read only after that step has finished
    (sk,) = [t for t in plan_of(lambda a, b: a @ (b + b), z(16, 4096), z(4096, 1024)).steps if t.kernel == "gemm_skinny"]
    assert sk.ints[7] == 0
    # 4 column blocks of 256: K split for two CTAs per SM (74 ranges wanted, 64-row multiples)
    assert kc == 64 and p.buffers[s.bufs[3][0]].nbytes == (4096 // 64) * 16 * 1024 * 4
    assert plan_of(mm, z(17, 4096), z(4096, 1024)).steps[0].kernel == "gemm_bf16"
    assert plan_of(mm_bt, z(8, 4096), z(1024, 4096)).steps[0].kernel == "gemm_bf16"
