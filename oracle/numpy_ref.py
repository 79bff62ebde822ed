"""NumPy restatement of the reference's CPU semantics for each configuration.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Dtype behaviour is the NumPy + ml_dtypes behaviour of a direct call: a bf16
matmul returns float32, elementwise bf16 ops round to bf16 per op.  Callers
compare the device result against these outputs after casting both to
float32, with the tolerances of the benchmark definition (1e-5 relative for
fp32 elementwise/reduction, 2e-2 for bf16 matmul paths, exact for indices).
"""

import contextlib

import ml_dtypes
import numpy as np

bfloat16 = np.dtype(ml_dtypes.bfloat16)


@contextlib.contextmanager
def fp32_accumulated_bf16_sums():
    """Run a kernel body's direct call with ``np.sum`` over bf16 accumulated in
    float32 (result rounded to bf16 once).

    NumPy reduces an ml_dtypes bf16 array strictly in order with a bf16
    rounding after every add, so a long sum stagnates once its ulp exceeds
    twice the addend (1000 x 0.2 sums to 64).  The traced ``reduce`` leaves the
    accumulation order open and the device kernels accumulate in fp32, so
    long bf16 reductions (the decode softmax over a KV cache,
    ``examples/models/qwen3/kernels/attention.py:141-143``) are compared against
    the direct call with this one change.  Every other op of the body runs as
    in the plain direct call."""
    plain = np.sum

    def sum32(a, axis=None, dtype=None, out=None, keepdims=False, **kw):
        arr = np.asarray(a)
        if arr.dtype == bfloat16 and dtype is None and out is None:
            return plain(arr.astype(np.float32), axis=axis, keepdims=keepdims, **kw).astype(bfloat16)
        return plain(a, axis=axis, dtype=dtype, out=out, keepdims=keepdims, **kw)

    np.sum = sum32
    try:
        yield
    finally:
        np.sum = plain


def softmax(x):
    """Row softmax, as ``tests/kernels/softmax.py:7-10`` of the reference."""
    m = np.max(x, axis=-1, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=-1, keepdims=True)


def rmsnorm(x, w, eps):
    """``examples/models/qwen3_embedding/kernels/rmsnorm.py:4-16``: fp32 compute."""
    dt = x.dtype
    xf = x.astype(np.float32)
    ms = np.mean(np.square(xf), axis=-1, keepdims=True)
    return ((xf / np.sqrt(ms + eps)) * w.astype(np.float32)).astype(dt)


def residual_rmsnorm(x, r, w, eps=1e-6):
    """Residual add (``examples/models/qwen3/kernels/transformer_layer.py:60``) then RMSNorm."""
    return rmsnorm(x + r, w, eps)


def matmul(a, b):
    """``np.matmul`` of two bf16 arrays; NumPy returns float32 (fp32 accumulate)."""
    return np.matmul(a.astype(np.float32), b.astype(np.float32))


def argmax(x, axis=-1):
    """First-occurrence argmax (``core/ops/reduce.py:227-311``), int32 like the trace."""
    return np.argmax(x, axis=axis).astype(np.int32)


def linear_attention_recurrent(q, k, v, chunk=64):
    """Causal linear attention, one chunk at a time with a running fp32 state.

    out_t = phi(q_t) . S_t / (phi(q_t) . z_t) with S_t = sum_{s<=t} phi(k_s) v_s^T,
    z_t = sum_{s<=t} phi(k_s), phi = elu + 1.  This is the per-step state update of
    ``examples/linear_attention/deltanet.py:100-128`` restated with the linear
    attention update rule, processed ``chunk`` steps at a time: inside a chunk the
    causal part is an explicit lower-triangular product, across chunks the state
    carries the history.  Output has q's dtype.
    """
    B, H, T, D = q.shape
    phi = lambda t: np.where(t > 0, t + 1.0, np.exp(np.minimum(t, 0.0))).astype(np.float32)  # noqa: E731
    qf, kf, vf = phi(q.astype(np.float32)), phi(k.astype(np.float32)), v.astype(np.float32)
    out = np.empty((B, H, T, D), dtype=np.float32)
    tri = np.tril(np.ones((chunk, chunk), dtype=np.float32))
    S = np.zeros((B, H, D, D), dtype=np.float32)
    z = np.zeros((B, H, D), dtype=np.float32)
    for c0 in range(0, T, chunk):
        qc, kc, vc = qf[:, :, c0 : c0 + chunk], kf[:, :, c0 : c0 + chunk], vf[:, :, c0 : c0 + chunk]
        sc = np.einsum("bhid,bhjd->bhij", qc, kc) * tri
        num = np.einsum("bhij,bhjd->bhid", sc, vc) + np.einsum("bhid,bhde->bhie", qc, S)
        den = sc.sum(-1) + np.einsum("bhid,bhd->bhi", qc, z)
        out[:, :, c0 : c0 + chunk] = num / den[..., None]
        S = S + np.einsum("bhjd,bhje->bhde", kc, vc)
        z = z + kc.sum(axis=2)
    return out.astype(q.dtype)


def rope_tables(seq_len, head_dim, theta):
    """``examples/models/qwen3_embedding/kernels/rope.py:4-31`` (cos/sin of S x D/2)."""
    inv = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    f = np.outer(np.arange(seq_len, dtype=np.float32), inv)
    return np.cos(f).astype(np.float32), np.sin(f).astype(np.float32)


def _rope(x, cos, sin):
    """Half-split rotation of ``rope.py:34-57``; x (B,S,H,D), tables (S, D/2).

    With bf16 operands every product and sum is rounded to bf16, as the
    NumPy/ml_dtypes direct call of the kernel body does.
    """
    h = x.shape[-1] // 2
    c, s = cos[None, :, None, :], sin[None, :, None, :]
    x0, x1 = x[..., :h], x[..., h:]
    if x.dtype == bfloat16 and cos.dtype == bfloat16:
        f = lambda a: a.astype(np.float32)  # noqa: E731
        r = lambda a: a.astype(bfloat16)  # noqa: E731
        lo = r(f(r(f(x0) * f(c))) - f(r(f(x1) * f(s))))
        hi = r(f(r(f(x0) * f(s))) + f(r(f(x1) * f(c))))
        return np.concatenate([lo, hi], axis=-1)
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)


def llama_layer(x, w, n_heads, n_kv_heads, head_dim, eps, theta, heads=None):
    """One Llama decoder layer (TP=1 view), reference-idiom dtypes.

    Follows ``examples/models/qwen3_embedding/kernels/transformer_layer.py:8-83``
    with ``attention.py:9-105`` (no q/k norm: Llama), ``ffn.py:11-46`` (SwiGLU)
    and ``softmax.py`` (fp32 softmax cast back).  ``w`` holds full weights
    ``qkv, o, gate, up, down, ln1, ln2`` used as ``x @ W``.  Matmuls accumulate
    in fp32 and round to bf16, elementwise bf16 ops round per op, like the
    NumPy/ml_dtypes direct call of the traced kernel.

    ``heads`` restricts attention to a subset of query heads (bounded CPU
    samples); the o-projection then only sums those heads' contributions, so
    the result is only comparable through ``llama_layer_attention_heads``.
    """
    bf = bfloat16
    B, S, Hd = x.shape
    h = rmsnorm(x, w["ln1"], eps)
    qkv = np.matmul(h.astype(np.float32), w["qkv"].astype(np.float32)).astype(bf)
    nq, nkv = n_heads * head_dim, n_kv_heads * head_dim
    q = qkv[..., :nq].reshape(B, S, n_heads, head_dim)
    k = qkv[..., nq : nq + nkv].reshape(B, S, n_kv_heads, head_dim)
    v = qkv[..., nq + nkv :].reshape(B, S, n_kv_heads, head_dim)
    cos, sin = (t.astype(bf) for t in rope_tables(S, head_dim, theta))
    q = _rope(q, cos, sin).astype(bf)
    k = _rope(k, cos, sin).astype(bf)
    rep = n_heads // n_kv_heads
    mask = np.triu(np.ones((S, S), dtype=np.float32) * -10000.0, k=1).astype(bf).astype(np.float32)
    attn = np.zeros((B, S, n_heads, head_dim), dtype=bf)
    sel = range(n_heads) if heads is None else heads
    scale = np.float32(1.0 / np.sqrt(head_dim))
    for b in range(B):
        for hh in sel:
            qh = q[b, :, hh].astype(np.float32)
            kh = k[b, :, hh // rep].astype(np.float32)
            vh = v[b, :, hh // rep].astype(np.float32)
            sc = (qh @ kh.T).astype(bf).astype(np.float32)
            sc = (sc * scale).astype(bf).astype(np.float32)  # trace: divide by sqrt(d) in bf16
            sc = (sc + mask).astype(bf).astype(np.float32)
            p = softmax(sc).astype(bf).astype(np.float32)
            attn[b, :, hh] = (p @ vh).astype(bf)
    o = np.matmul(attn.reshape(B, S, Hd).astype(np.float32), w["o"].astype(np.float32)).astype(bf)
    h1 = (x.astype(np.float32) + o.astype(np.float32)).astype(bf)
    h2 = rmsnorm(h1, w["ln2"], eps)
    gate = np.matmul(h2.astype(np.float32), w["gate"].astype(np.float32)).astype(bf).astype(np.float32)
    up = np.matmul(h2.astype(np.float32), w["up"].astype(np.float32)).astype(bf).astype(np.float32)
    act = (gate / (1.0 + np.exp(-gate))).astype(bf).astype(np.float32) * up
    d = np.matmul(act.astype(bf).astype(np.float32), w["down"].astype(np.float32)).astype(bf)
    return (h1.astype(np.float32) + d.astype(np.float32)).astype(bf)


# -- simulated collectives: identical data on every rank ----------------------
def all_reduce_identical(data, world, reduce_op=np.add):
    """Reference CPU semantics (``core/ops/collectives.py:62-84``)."""
    if reduce_op is np.add:
        return data * world
    if reduce_op is np.multiply:
        return data**world
    return data.copy()


def all_gather_identical(data, world, dim):
    """Reference CPU semantics (``core/ops/collectives.py:17-31``): tile along ``dim``."""
    return np.tile(data, tuple(world if i == dim else 1 for i in range(data.ndim)))


def reduce_scatter_identical(data, world, dim):
    """Reference CPU semantics (``core/ops/collectives.py:120-145``): sum, then rank 0's block."""
    return np.take(data * world, range(data.shape[dim] // world), axis=dim)


# -- top-k ---------------------------------------------------------------------
def topk(x, k, is_ascend=False):
    """Last-axis top-k with a total order: values largest first (smallest first
    when ``is_ascend``), ties by the lower index, indices as uint32.

    The reference's CPU implementation (``core/ops/nn.py:22-62``) selects the
    same set with ``np.argpartition`` and orders it with ``np.argsort``, whose
    default sort leaves the order of equal values unspecified; its device path
    is the HLO TopK (``nn.py:65-152``), which keeps equal values in index order.
    This restatement fixes that order, so that it agrees with the reference
    CPU result wherever the values are distinct, and states the tie order the
    device kernel must reproduce bit for bit (NaN and the sign of zero are
    outside it: the kernel orders those by bit pattern)."""
    wide = x.astype(np.float64) if (x.dtype.kind == "f" or x.dtype == bfloat16) else x.astype(np.int64)
    idx = np.argsort(wide if is_ascend else -wide, axis=-1, kind="stable")[..., :k]
    return np.take_along_axis(x, idx, axis=-1), idx.astype(np.uint32)


# -- convolution ------------------------------------------------------------------
def conv_nd(x, w, bias=None, stride=1, padding=0, dilation=1):
    """N-d cross-correlation, NC-spatial layout (reference ``core/ops/conv.py``:
    CPU ``:133-228``, traced attributes ``:230-312``).  Accumulated in float64
    as a sum over kernel offsets of shifted, strided input slices times the
    weight; returns float32 (what the reference's fp32 direct call returns)."""
    n = x.ndim - 2
    st = (stride,) * n if np.isscalar(stride) else tuple(stride)
    pd = (padding,) * n if np.isscalar(padding) else tuple(padding)
    dl = (dilation,) * n if np.isscalar(dilation) else tuple(dilation)
    xf = np.pad(x.astype(np.float64), ((0, 0), (0, 0)) + tuple((p, p) for p in pd))
    wf = w.astype(np.float64)
    ks = w.shape[2:]
    out_sp = tuple((xf.shape[2 + i] - dl[i] * (ks[i] - 1) - 1) // st[i] + 1 for i in range(n))
    y = np.zeros((x.shape[0], w.shape[0]) + out_sp)
    for off in np.ndindex(*ks):
        sl = tuple(slice(off[i] * dl[i], off[i] * dl[i] + st[i] * (out_sp[i] - 1) + 1, st[i]) for i in range(n))
        patch = xf[(slice(None), slice(None)) + sl]  # (B, C, *out)
        y += np.einsum("bc...,oc->bo...", patch, wf[(slice(None), slice(None)) + off])
    if bias is not None:
        y += bias.astype(np.float64).reshape((1, -1) + (1,) * n)
    return y.astype(np.float32)
