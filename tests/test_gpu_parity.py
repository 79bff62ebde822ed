"""Parity of the B200 path against the CPU oracle (NumPy direct-call semantics).

Each test traces a kernel body, plans it, runs it through libnkb's C ABI
(``DeviceKernel`` / ``baremetal_run_traced_kernel``) and compares with the
oracle on the same seeded inputs.  Tolerances: 1e-5 relative for fp32
elementwise/reduction work, 2e-2 relative for bf16 matmul paths, exact for
integer/index results.
"""

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200 import workloads as W
from oracle import numpy_ref as O
from tests.utils import BF16_RTOL, FP32_RTOL, assert_close, on_device, sum_abs_atol

BF16 = np.dtype(ml_dtypes.bfloat16)
pytestmark = pytest.mark.gpu


@pytest.mark.parametrize(
    "shape", [(4096, 4096), (7, 1000), (33, 128), (3, 9000), (2, 130), (1, 1), (5, 2000), (2000, 6000), (300, 8192)]
)
def test_softmax(shape):
    x = np.random.default_rng(1).standard_normal(shape, dtype=np.float32)
    got = on_device(W.softmax_kernel, x)
    assert_close(got, O.softmax(x), FP32_RTOL, atol=1e-7)


@pytest.mark.parametrize("rows,cols", [(16384, 4096), (5, 4096), (17, 1000), (3, 12288), (1, 64)])
def test_residual_rmsnorm(rows, cols):
    x, r, w = W.make_inputs("rmsnorm", seed=3, scale=1.0)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((rows, cols), dtype=np.float32)
    r = rng.standard_normal((rows, cols), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    got = on_device(W.residual_rmsnorm_kernel, x, r, w)
    assert_close(got, O.residual_rmsnorm(x, r, w, 1e-6), FP32_RTOL)


@pytest.mark.parametrize("rows,cols,res", [(16, 4096, True), (5, 2048, False), (3, 8192, True), (7, 1536, True),
                                           (8192, 4096, True)])
def test_residual_rmsnorm_bf16(rows, cols, res):
    """bf16 rows (the decoder layer's norms) on the 16-byte-vector kernel; the
    direct call rounds the residual sum and the result to bf16, so the device
    result may differ by one bf16 unit in the last place."""
    rng = np.random.default_rng(26)
    x = rng.standard_normal((rows, cols), dtype=np.float32).astype(BF16)
    r = rng.standard_normal((rows, cols), dtype=np.float32).astype(BF16)
    w = rng.uniform(0.5, 1.5, cols).astype(BF16)
    if res:
        got = on_device(W.residual_rmsnorm_kernel, x, r, w)
        want = W.residual_rmsnorm_kernel(x, r, w)
    else:
        got = on_device(lambda a, g: W.rmsnorm(a, g, 1e-6), x, w)
        want = W.rmsnorm(x, w, 1e-6)
    assert got.dtype == BF16
    assert_close(got, want, 2**-7, atol=2**-7)


@pytest.mark.parametrize("m,k,n", [(256, 512, 256), (8192, 8192, 8192), (300, 200, 264), (128, 64, 256), (1000, 4096, 1000),
                                   (8, 4096, 6144), (1, 4096, 4096), (5, 12288, 1000), (16, 200, 264), (3, 64, 8)])
def test_matmul_bf16(m, k, n):
    """Tiles of 128 x 256 on tcgen05; products with few tiles split their K range
    across the SMs; at most 16 rows (decode rows against a weight matrix, ragged
    K ranges and column blocks) run on the skinny mma.sync kernel."""
    rng = np.random.default_rng(5)
    a = (rng.standard_normal((m, k), dtype=np.float32) * 0.02).astype(BF16)
    b = (rng.standard_normal((k, n), dtype=np.float32) * 0.02).astype(BF16)
    got = on_device(W.matmul_kernel, a, b)
    assert got.dtype == BF16
    assert_close(got, O.matmul(a, b), BF16_RTOL)


@pytest.mark.parametrize("layout", ["a_t", "b_t", "both_t"])
@pytest.mark.parametrize("m,k,n", [(1000, 512, 776), (4096, 1024, 2048), (200, 64, 128)])
def test_matmul_bf16_transposed_operands(layout, m, k, n):
    """M-major A (A stored K x M) and K-major B (B stored N x K) on the tensor cores."""
    rng = np.random.default_rng(17)
    a = (rng.standard_normal((m, k), dtype=np.float32) * 0.05).astype(BF16)
    b = (rng.standard_normal((k, n), dtype=np.float32) * 0.05).astype(BF16)
    at, bt = np.ascontiguousarray(a.T), np.ascontiguousarray(b.T)
    kern = {
        "a_t": lambda x, y: x.T @ y,
        "b_t": lambda x, y: x @ y.T,
        "both_t": lambda x, y: x.T @ y.T,
    }[layout]
    args = {"a_t": (at, b), "b_t": (a, bt), "both_t": (at, bt)}[layout]
    got = on_device(kern, *args)
    assert_close(got, O.matmul(a, b), BF16_RTOL)


@pytest.mark.parametrize("b,m,k,n", [(32, 2048, 2048, 2048), (3, 130, 72, 200)])
def test_bmm_bf16(b, m, k, n):
    rng = np.random.default_rng(6)
    a = (rng.standard_normal((b, m, k), dtype=np.float32) * 0.02).astype(BF16)
    bb = (rng.standard_normal((b, k, n), dtype=np.float32) * 0.02).astype(BF16)
    got = on_device(W.bmm_kernel, a, bb)
    assert_close(got, O.matmul(a, bb), BF16_RTOL)


def test_matmul_fp32_simt():
    rng = np.random.default_rng(7)
    a = rng.standard_normal((70, 50), dtype=np.float32)
    b = rng.standard_normal((50, 90), dtype=np.float32)
    got = on_device(W.matmul_kernel, a, b)
    # each output is a 50-term dot product: bounded by the magnitudes of its terms
    assert_close(got, a @ b, FP32_RTOL, atol=FP32_RTOL * (np.abs(a) @ np.abs(b)))


def test_elementwise_chain_broadcast():
    def k(x, y, z):
        t = np.exp(x - y[None, :]) * 0.5 + np.tanh(z[:, None])
        return np.where(t > 1.0, t, -t) / (1.0 + np.abs(x))

    rng = np.random.default_rng(8)
    x = rng.standard_normal((37, 65), dtype=np.float32)
    y = rng.standard_normal((65,), dtype=np.float32)
    z = rng.standard_normal((37,), dtype=np.float32)
    assert_close(on_device(k, x, y, z), k(x, y, z), 1e-5)


@pytest.mark.parametrize("dtype,shape", [(np.float32, (64, 256)), (np.float32, (3, 5, 96)), (BF16, (40, 512)),
                                         (np.float32, (7, 13))])
def test_elementwise_chain_register_reuse(dtype, shape):
    """Six inputs, values read again several instructions later (from the
    shared-memory register file, not the accumulator), a select on a
    recomputed value, a result that is not the last instruction's; row-run
    kernel (8- and 4-element runs) and the generic kernel (13 columns)."""

    def k(a, b, c, d, e, f):
        t = a * b + c
        u = np.where(t > d, t, e * t)
        return u - f * a + np.exp(-u) * b, t

    rng = np.random.default_rng(24)
    args = [rng.standard_normal(shape, dtype=np.float32).astype(dtype) for _ in range(6)]
    got = on_device(k, *args)
    want = k(*args)
    for g, w in zip(got, want):
        if dtype == BF16:
            assert_close(g, w, BF16_RTOL)
        else:
            assert_close(g, w, FP32_RTOL)


def test_argmax_exact():
    def k(x):
        return np.argmax(x, axis=-1)

    rng = np.random.default_rng(9)
    x = rng.standard_normal((64, 1000), dtype=np.float32)
    x[3, 10] = x[3, 20] = 100.0  # tie: first occurrence wins
    got = on_device(k, x)
    np.testing.assert_array_equal(got, O.argmax(x))


def test_transpose_exact():
    def k(x):
        return np.transpose(x, (1, 0, 2)).copy()

    x = np.arange(5 * 7 * 3, dtype=np.int32).reshape(5, 7, 3)
    np.testing.assert_array_equal(on_device(k, x), np.transpose(x, (1, 0, 2)))


def test_take_exact():
    def k(x, idx):
        return np.take(x, idx, axis=0)

    x = np.random.default_rng(10).standard_normal((50, 33), dtype=np.float32)
    idx = np.array([3, 0, 49, 7, 7], dtype=np.int32)
    np.testing.assert_array_equal(on_device(k, x, idx), x[idx])


def test_reductions():
    def k(x):
        return np.sum(x, axis=0), np.max(x, axis=1), np.mean(x)

    x = np.random.default_rng(11).standard_normal((300, 77), dtype=np.float32)
    s, m, mu = on_device(k, x)
    assert_close(s, x.sum(0), FP32_RTOL, atol=sum_abs_atol(x, axis=0))
    np.testing.assert_array_equal(m, x.max(1))
    assert_close(mu, np.mean(x), FP32_RTOL, atol=FP32_RTOL * float(np.mean(np.abs(x))))


@pytest.mark.parametrize("batch,seq", [(2, 128), (1, 512)])
def test_llama_layer_tp1(batch, seq):
    s = W.LayerShape(batch=batch, seq=seq, hidden=512, n_heads=8, n_kv_heads=2, head_dim=64, ffn=1024)
    full = W.layer_weights(s, seed=1)
    shard = W.shard_layer_weights(full, s, 0, 1)
    x = np.random.default_rng(12).standard_normal((batch, seq, s.hidden), dtype=np.float32).astype(BF16)
    args, kw = W.layer_args(x, shard, s, 1)
    got = on_device(W.llama_decoder_layer_kernel, *args, **kw)
    want = O.llama_layer(x, full, s.n_heads, s.n_kv_heads, s.head_dim, s.eps, s.theta)
    assert got.dtype == BF16
    assert_close(got, want, BF16_RTOL)


def _run_layer(x, shard, s, world=1):
    """Plan and run one layer shard through DeviceKernel; returns (y, kernel counts)."""
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    args, kw = W.layer_args(x, shard, s, world)
    k = DeviceKernel.compile_and_load(W.llama_decoder_layer_kernel, *args, name="layer_test", is_spmd=False, **kw)
    names = [t["name"] for t in k.model_ref.io["inputs"]]
    outs = k(inputs={n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(names, args)})
    return next(iter(outs.values())).numpy(), k.model_ref.io["kernels"], k.model_ref.num_launches


# The benchmarked layer's kernels at a reduced size: head_dim 128 sends
# attention to the tcgen05 flash kernel and runs the RoPE epilogue of the QKV
# GEMM on 128-wide heads; the SwiGLU and residual epilogues run on their own
# GEMMs.  Seven launches: RMSNorm, QKV+RoPE, attention, O+residual,
# RMSNorm, gate/up+SwiGLU, down+residual.
@pytest.mark.parametrize("batch,seq,hidden,nq,nkv,ffn", [(2, 256, 1024, 8, 2, 2048), (1, 384, 2048, 16, 4, 2816)])
def test_llama_layer_head_dim_128(batch, seq, hidden, nq, nkv, ffn):
    s = W.LayerShape(batch=batch, seq=seq, hidden=hidden, n_heads=nq, n_kv_heads=nkv, head_dim=128, ffn=ffn)
    full = W.layer_weights(s, seed=21)
    x = np.random.default_rng(22).standard_normal((batch, seq, hidden), dtype=np.float32).astype(BF16)
    got, kinds, launches = _run_layer(x, W.shard_layer_weights(full, s, 0, 1), s)
    assert launches == 7 and kinds.get("flash_attn") == 1 and kinds.get("gemm_bf16") == 4, kinds
    want = O.llama_layer(x, full, s.n_heads, s.n_kv_heads, s.head_dim, s.eps, s.theta)
    assert got.dtype == BF16
    assert_close(got, want, BF16_RTOL)


def test_llama_layer_benchmark_shape_causal_prefix():
    """The benchmarked configuration itself (batch 4 x 2048 tokens, hidden 4096,
    32q/8kv x 128, FFN 14336) on the device; by causality the first 256 output
    tokens of sequence 0 depend only on its first 256 input tokens, so they are
    compared with the oracle's layer on that prefix (as bench.py does at every
    GPU count)."""
    s = W.LayerShape()
    full = W.layer_weights(s, seed=0)
    x = np.random.default_rng(500).standard_normal((s.batch, s.seq, s.hidden), dtype=np.float32).astype(BF16)
    got, kinds, launches = _run_layer(x, W.shard_layer_weights(full, s, 0, 1), s)
    assert launches == 7 and kinds.get("flash_attn") == 1, kinds
    want = O.llama_layer(x[:1, :256], full, s.n_heads, s.n_kv_heads, s.head_dim, s.eps, s.theta)
    assert_close(got[:1, :256], want, BF16_RTOL)
    assert np.all(np.isfinite(got.astype(np.float32)))


def _attention_body(q, k, v, n_rep):
    B, S, H, D = q.shape
    if n_rep > 1:
        k = np.repeat(k, n_rep, axis=2)
        v = np.repeat(v, n_rep, axis=2)
    q, k, v = q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3)
    scores = (q @ k.transpose(0, 1, 3, 2)) / np.sqrt(D)
    mask = np.triu(np.ones((S, S)) * -10000.0, k=1).astype(scores.dtype)
    scores = scores + mask[None, None, :, :]
    x = scores.astype(np.float32)
    e = np.exp(x - np.max(x, axis=-1, keepdims=True))
    p = (e / np.sum(e, axis=-1, keepdims=True)).astype(scores.dtype)
    return (p @ v).transpose(0, 2, 1, 3)


# head_dim 128 runs the tcgen05 kernel (two 128-row tiles per CTA): full tiles,
# a ragged last pair, a second tile with 2 valid rows, an empty second tile, and
# a long sequence with widely spread scores (qscale) so the running maximum is
# raised and O rescaled; head_dim 64 the mma.sync kernel.
@pytest.mark.parametrize(
    "B,S,H,Hkv,D,qscale",
    [(2, 256, 8, 2, 128, 1.0), (1, 200, 4, 4, 64, 1.0), (1, 1000, 2, 1, 128, 1.0), (4, 130, 2, 2, 128, 1.0),
     (1, 64, 2, 1, 128, 1.0), (1, 2048, 4, 1, 128, 4.0)],
)
def test_flash_attention_gqa_causal(B, S, H, Hkv, D, qscale):
    rng = np.random.default_rng(13)
    q = (qscale * rng.standard_normal((B, S, H, D), dtype=np.float32)).astype(BF16)
    k = rng.standard_normal((B, S, Hkv, D), dtype=np.float32).astype(BF16)
    v = rng.standard_normal((B, S, Hkv, D), dtype=np.float32).astype(BF16)
    n_rep = H // Hkv

    def kern(q, k, v):
        return _attention_body(q, k, v, n_rep)

    got = on_device(kern, q, k, v)
    # oracle: fp32 attention on the same bf16 inputs
    qf, kf, vf = (t.astype(np.float32) for t in (q, k, v))
    kf, vf = np.repeat(kf, n_rep, axis=2), np.repeat(vf, n_rep, axis=2)
    s = np.einsum("bqhd,bkhd->bhqk", qf, kf) / np.sqrt(D)
    s = s + np.triu(np.full((S, S), -np.inf, np.float32), k=1)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    want = np.einsum("bhqk,bkhd->bqhd", p, vf)
    assert_close(got, want, BF16_RTOL)


@pytest.mark.parametrize("tokens,hidden,ffn", [(256, 512, 1024), (300, 256, 320)])
def test_swiglu_ffn(tokens, hidden, ffn):
    def ffn_kernel(x, gate_up, down):
        gate, up = np.split(x @ gate_up, 2, axis=-1)
        return (W.silu(gate) * up) @ down

    rng = np.random.default_rng(14)
    x = rng.standard_normal((tokens, hidden), dtype=np.float32).astype(BF16)
    gu = (rng.standard_normal((hidden, 2 * ffn), dtype=np.float32) * 0.02).astype(BF16)
    dn = (rng.standard_normal((ffn, hidden), dtype=np.float32) * 0.02).astype(BF16)
    got = on_device(ffn_kernel, x, gu, dn)
    f = lambda t: t.astype(np.float32)  # noqa: E731
    r = lambda t: t.astype(BF16)  # noqa: E731
    h = r(f(x) @ f(gu))
    g, u = f(h[:, :ffn]), f(h[:, ffn:])
    act = r(f(r(g * f(r(1.0 / f(r(1.0 + f(r(np.exp(-g))))))))) * u)
    want = f(act) @ f(dn)
    assert_close(got, want, BF16_RTOL)


# head_dim 32 takes the generic lowering; the others the tensor-core kernel:
# one segment, a 64-token tail block, a single partial block, several segments
# (with a tail segment of one partial block), and 96 heads (one segment each).
@pytest.mark.parametrize(
    "shape",
    [(1, 2, 256, 32), (2, 3, 512, 128), (1, 2, 320, 128), (1, 1, 64, 128), (1, 2, 3072, 128),
     (1, 1, 2560, 128), (1, 1, 1088, 128), (2, 48, 256, 128)],
)
def test_chunked_linear_attention(shape):
    rng = np.random.default_rng(15)
    q, k, v = (rng.standard_normal(shape, dtype=np.float32).astype(BF16) for _ in range(3))
    got = on_device(W.chunked_linear_attention_kernel, q, k, v)
    want = O.linear_attention_recurrent(q, k, v)
    assert_close(got, want, BF16_RTOL)


def test_chunked_linear_attention_benchmark_shape():
    """The benchmarked input (8, 16, 4096, 128) on the device; two (batch, head)
    pairs of it (first and last) against the recurrent oracle, every pair
    finite."""
    q, k, v = W.make_inputs("linattn", seed=600)
    got = on_device(W.chunked_linear_attention_kernel, q, k, v)
    assert got.shape == q.shape and got.dtype == BF16
    for b, h in ((0, 0), (7, 15)):
        sl = (slice(b, b + 1), slice(h, h + 1))
        want = O.linear_attention_recurrent(q[sl], k[sl], v[sl])
        assert_close(got[sl], want, BF16_RTOL)
    assert np.all(np.isfinite(got.astype(np.float32)))


@pytest.mark.parametrize(
    "shape,k,dtype,asc",
    [
        ((64, 1000), 1, np.float32, False),
        ((64, 1000), 8, np.float32, True),
        ((3, 151936), 4, BF16, False),  # a Qwen3 vocabulary row: longer than the shared-memory stage
        ((17, 49152), 3, np.float32, False),  # the longest staged row
        ((2, 4096), 64, np.float32, False),
        ((5, 7), 7, np.int32, False),
        ((1, 1), 1, np.float32, False),
        ((300, 130), 5, np.float16, True),
        ((8, 32768), 16, BF16, False),  # 16-key lists, 8 parts per row
        ((4, 65536), 32, np.float16, True),  # 32-key lists, 16 parts
        ((6, 20000), 9, np.int32, False),  # ties in every part, 4 parts
        ((128, 151936), 8, BF16, False),  # the sampling benchmark: candidates ranked in shared memory
        ((4, 151936), 8, np.int32, False),  # thousands of ties above the threshold: the list path
        ((2, 3000), 8, BF16, True),  # one part, warps without a full share of the row
    ],
)
def test_topk_exact(shape, k, dtype, asc):
    from nkipy_b200.core.ops import nn

    def kern(x):
        return nn.topk(x, k, axis=-1, is_ascend=asc)

    rng = np.random.default_rng(13)
    if np.dtype(dtype).kind == "i":
        x = rng.integers(-50, 50, shape).astype(dtype)  # many ties: lower index first
    else:
        x = rng.standard_normal(shape, dtype=np.float32).astype(dtype)  # bf16/f16 rounding makes ties too
    vals, idx = on_device(kern, x)
    want_v, want_i = O.topk(x, k, is_ascend=asc)
    np.testing.assert_array_equal(idx, want_i)
    np.testing.assert_array_equal(vals.view(np.uint8), want_v.view(np.uint8))


def test_greedy_sampling_single_device():
    B, S, H, V = 4, 8, 512, 32000
    rng = np.random.default_rng(14)
    h = rng.standard_normal((B, S, H), dtype=np.float32).astype(BF16)
    nw = rng.uniform(0.5, 1.5, H).astype(BF16)
    lm = (rng.standard_normal((H, V), dtype=np.float32) * 0.05).astype(BF16)
    ids = on_device(W.greedy_sampling_kernel, h, nw, lm, max_batch_size=B).reshape(-1).astype(np.int64)
    logits = W.qk_rmsnorm(h, nw, 1e-6)[:, -1, :].astype(np.float32) @ lm.astype(np.float32)
    best = logits.max(axis=1)
    assert np.all((ids >= 0) & (ids < V))
    # the chosen token holds the largest logit, up to the bf16 rounding of the device's logits
    assert np.all(logits[np.arange(B), ids] >= best - (2.0**-7 * np.abs(best) + 1e-6))



@pytest.mark.parametrize(
    "n,x_shape,w_shape,kw,dtype,bias",
    [
        (2, (2, 16, 20, 24), (32, 16, 3, 3), dict(stride=1, padding=1), BF16, True),  # tensor-core GEMM
        (2, (3, 3, 17, 13), (5, 3, 4, 2), dict(stride=(2, 1), padding=(1, 3)), np.float32, True),
        (2, (1, 2, 9, 9), (3, 2, 3, 3), dict(stride=1, padding=2, dilation=2), np.float32, False),
        (3, (1, 2, 6, 7, 8), (4, 2, 2, 3, 2), dict(stride=(1, 2, 1), padding=1), np.float32, True),
        # bf16 with the last output axis a multiple of 8: the 16-byte window kernel
        (2, (2, 8, 32, 32), (16, 8, 3, 3), dict(stride=2, padding=1), BF16, True),  # stride 2
        (2, (1, 4, 24, 24), (8, 4, 3, 3), dict(stride=1, padding=2, dilation=2), BF16, False),  # dilation 2
        (3, (1, 2, 6, 7, 16), (4, 2, 2, 3, 3), dict(stride=(1, 2, 1), padding=1), BF16, True),  # 3-D
        # 3x3 "same" windows (stride 1, padding 1) on rows of 8k: the shifted-chunk kernel
        (2, (3, 3, 5, 8), (4, 3, 3, 3), dict(stride=1, padding=1), BF16, True),  # odd channels, one chunk
        (2, (1, 5, 1, 16), (2, 5, 3, 3), dict(stride=1, padding=1), BF16, False),  # one row
        (2, (2, 6, 7, 40), (8, 6, 3, 3), dict(stride=1, padding=1), BF16, True),  # five chunks per row
    ],
)
def test_convolution(n, x_shape, w_shape, kw, dtype, bias):
    from nkipy_b200.core import ops as OPS

    conv = OPS.conv2d if n == 2 else OPS.conv3d
    rng = np.random.default_rng(16)
    x = rng.standard_normal(x_shape, dtype=np.float32).astype(dtype)
    w = (rng.standard_normal(w_shape, dtype=np.float32) * 0.1).astype(dtype)
    b = rng.standard_normal(w_shape[0], dtype=np.float32).astype(dtype)
    if bias:
        got = on_device(lambda x, w, b: conv(x, w, b, **kw), x, w, b)
    else:
        got = on_device(lambda x, w: conv(x, w, **kw), x, w)
    want = O.conv_nd(x, w, b if bias else None, **kw)
    if dtype == BF16:
        assert_close(got, want, BF16_RTOL)
    else:
        # each output is a dot product over the window: bounded by its terms' magnitudes
        mag = O.conv_nd(np.abs(x), np.abs(w), np.abs(b) if bias else None, **kw)
        assert_close(got, want, FP32_RTOL, atol=FP32_RTOL * mag)


# Layout moves whose innermost axis changes run on the TMA tile-transpose
# kernel (2- and 4-byte elements, 16-byte aligned strides); the others on the
# elementwise copy.  Bit-exact either way.
@pytest.mark.parametrize(
    "shape,perm,dtype",
    [
        ((8192, 8192), (1, 0), np.float32),
        ((8192, 8192), (1, 0), BF16),
        ((1000, 776), (1, 0), np.float32),  # ragged edges in both axes
        ((776, 1000), (1, 0), BF16),
        ((64, 128, 256), (2, 0, 1), np.float32),  # two axes merge into R
        ((8, 16, 24, 40), (3, 2, 1, 0), np.float32),  # two batch axes, R shorter than a tile
        ((4, 128, 2000), (0, 2, 1), np.int32),
        ((2, 3, 4, 32, 64), (2, 1, 0, 4, 3), np.float16),  # three batch axes
        ((3, 100, 36), (0, 2, 1), BF16),  # 72-byte rows: elementwise copy
        ((300, 1000), (1, 0), np.int8),  # 1-byte elements: elementwise copy
    ],
)
def test_transpose_layout_move_exact(shape, perm, dtype):
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    rng = np.random.default_rng(23)
    if np.dtype(dtype).kind in "iu":
        x = rng.integers(-100, 100, shape).astype(dtype)
    else:
        x = rng.standard_normal(shape, dtype=np.float32).astype(dtype)

    def kern(a):
        return np.transpose(a, perm)

    k = DeviceKernel.compile_and_load(kern, x, name="transpose_test", is_spmd=False)
    aligned = np.dtype(dtype).itemsize in (2, 4) and shape != (3, 100, 36)
    assert k.model_ref.io["kernels"] == ({"transpose_tiles": 1} if aligned else {"ew": 1}), k.model_ref.io["kernels"]
    got = next(iter(k(inputs={"a": DeviceTensor.from_numpy(x, name="a")}).values())).numpy()
    want = np.ascontiguousarray(np.transpose(x, perm))
    assert got.shape == want.shape
    np.testing.assert_array_equal(got.view(np.uint8), want.view(np.uint8))


def test_convolution_bf16_window_kernel_64bit_indices(monkeypatch):
    """The 16-byte window kernel's 64-bit index instantiation (taken for very
    large inputs) on a small case, through its switch NKB_IM2COL_INDEX64."""
    from nkipy_b200.core import ops as OPS

    monkeypatch.setenv("NKB_IM2COL_INDEX64", "1")
    rng = np.random.default_rng(25)
    x = rng.standard_normal((2, 8, 32, 32), dtype=np.float32).astype(BF16)
    w = (rng.standard_normal((16, 8, 3, 3), dtype=np.float32) * 0.1).astype(BF16)
    got = on_device(lambda x, w: OPS.conv2d(x, w, stride=2, padding=1), x, w)
    assert_close(got, O.conv_nd(x, w, None, stride=2, padding=1), BF16_RTOL)
