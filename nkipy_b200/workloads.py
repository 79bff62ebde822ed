"""The five benchmark workloads as NKIPy kernel bodies (plain NumPy functions).

Each body is written in the reference's kernel idiom, so it runs on CPU by a
direct call and traces unchanged:

* ``softmax_kernel``: ``tests/kernels/softmax.py:7-10`` / ``README.md:125-128``;
* ``residual_rmsnorm_kernel``: residual add (``examples/models/qwen3/kernels/
  transformer_layer.py:60``) + RMSNorm (``examples/models/qwen3_embedding/
  kernels/rmsnorm.py:4-16``);
* ``matmul_kernel`` / ``bmm_kernel``: ``np.matmul`` (``core/ops/linalg.py:15``);
  NKIPy has no ``np.einsum`` so ``bmk,bkn->bmn`` is written as a batched matmul;
* ``chunked_linear_attention_kernel``: no reference body exists; this one
  follows the per-step state update idiom of ``examples/linear_attention/
  deltanet.py:74-128`` in chunked form (feature map elu+1, chunk 64, fp32
  running state, Katharopoulos normaliser);
* ``llama_decoder_layer_kernel``: the dense prefill layer of
  ``examples/models/qwen3_embedding/kernels/transformer_layer.py:8-83``
  (attention ``attention.py:9-105`` without the Qwen3 q/k norms, SwiGLU
  ``ffn.py:11-46``, RoPE ``rope.py:4-57``), tensor-parallel as in
  ``examples/models/qwen3/kernels/attention.py:61-64,150`` (local heads,
  all-reduce after the row-parallel projections).

``make_inputs(config, ...)`` builds the seeded synthetic inputs of each
configuration (shapes and distributions of the benchmark definition).
"""

from dataclasses import dataclass

import ml_dtypes
import numpy as np

from nkipy_b200.core.ops import collectives as cc

bfloat16 = np.dtype(ml_dtypes.bfloat16)


# ---------------------------------------------------------------------------
# 1. softmax
# ---------------------------------------------------------------------------
def softmax_kernel(x):
    exp_x = np.exp(x - np.max(x, axis=-1, keepdims=True))
    sum_x = np.sum(exp_x, axis=-1, keepdims=True)
    return exp_x / sum_x


# ---------------------------------------------------------------------------
# 2. residual add + RMSNorm
# ---------------------------------------------------------------------------
def rmsnorm(x, weight, eps):
    compute_dtype = np.float32
    original_dtype = x.dtype
    x = x.astype(compute_dtype)
    weight = weight.astype(compute_dtype)
    z = np.square(x)
    z = np.mean(z, axis=-1, keepdims=True)
    z = x / np.sqrt(z + eps)
    res = z * weight
    return res.astype(original_dtype)


def residual_rmsnorm_kernel(x, r, weight, eps=1e-6):
    return rmsnorm(x + r, weight, eps)


# ---------------------------------------------------------------------------
# 3. matmul / batched matmul
# ---------------------------------------------------------------------------
def matmul_kernel(a, b):
    return a @ b


def bmm_kernel(a, b):
    return np.matmul(a, b)


# ---------------------------------------------------------------------------
# 4. chunked causal linear attention
# ---------------------------------------------------------------------------
def elu_plus_one(x):
    # elu(x) + 1 == x + 1 for x > 0, exp(x) otherwise
    return np.where(x > 0, x + 1.0, np.exp(x))


def chunked_linear_attention_kernel(q, k, v, chunk=64):
    B, H, T, D = q.shape
    n_chunks = T // chunk
    phi_q = elu_plus_one(q.astype(np.float32)).reshape(B, H, n_chunks, chunk, D)
    phi_k = elu_plus_one(k.astype(np.float32)).reshape(B, H, n_chunks, chunk, D)
    vf = v.astype(np.float32).reshape(B, H, n_chunks, chunk, D)
    causal = np.tril(np.ones((chunk, chunk), dtype=np.float32))
    # per-chunk key/value state and key sum, then the exclusive prefix over chunks
    kv = np.matmul(phi_k.transpose(0, 1, 2, 4, 3), vf)  # (B,H,N,D,D)
    ksum = np.sum(phi_k, axis=3, keepdims=True)  # (B,H,N,1,D)
    state = np.cumsum(kv, axis=2) - kv
    zsum = np.cumsum(ksum, axis=2) - ksum
    scores = np.matmul(phi_q, phi_k.transpose(0, 1, 2, 4, 3)) * causal  # (B,H,N,C,C)
    num = np.matmul(scores, vf) + np.matmul(phi_q, state)
    den = np.sum(scores, axis=-1, keepdims=True) + np.sum(phi_q * zsum, axis=-1, keepdims=True)
    out = (num / den).reshape(B, H, T, D)
    return out.astype(q.dtype)


# ---------------------------------------------------------------------------
# 5. Llama decoder layer (tensor-parallel shard)
# ---------------------------------------------------------------------------
def softmax(x):
    original_dtype = x.dtype
    x = x.astype(np.float32)
    exp_x = np.exp(x - np.max(x, axis=-1, keepdims=True))
    return (exp_x / np.sum(exp_x, axis=-1, keepdims=True)).astype(original_dtype)


def rope(xq, xk, cos, sin):
    cos = np.expand_dims(cos, axis=(0, 2))
    sin = np.expand_dims(sin, axis=(0, 2))
    half = xq.shape[-1] // 2
    xq0, xq1 = xq[:, :, :, :half], xq[:, :, :, half:]
    xk0, xk1 = xk[:, :, :, :half], xk[:, :, :, half:]
    xq_out = np.concatenate([xq0 * cos - xq1 * sin, xq0 * sin + xq1 * cos], axis=-1)
    xk_out = np.concatenate([xk0 * cos - xk1 * sin, xk0 * sin + xk1 * cos], axis=-1)
    return xq_out, xk_out


def silu(x):
    return x * (1 / (1 + np.exp(-x)))


def llama_decoder_layer_kernel(
    x,
    input_norm_weight,
    qkv_weight,
    o_weight,
    post_norm_weight,
    gate_up_weight,
    down_weight,
    cos,
    sin,
    n_heads=32,
    n_kv_heads=8,
    head_dim=128,
    eps=1e-6,
    tp_world=1,
):
    B, S, _ = x.shape
    nq = n_heads // tp_world
    nkv = max(1, n_kv_heads // tp_world)
    n_rep = nq // nkv

    h = rmsnorm(x, input_norm_weight, eps)
    qkv = h @ qkv_weight
    q, k, v = np.split(qkv, [nq * head_dim, (nq + nkv) * head_dim], axis=-1)
    q = q.reshape(B, S, nq, head_dim)
    k = k.reshape(B, S, nkv, head_dim)
    v = v.reshape(B, S, nkv, head_dim)
    q, k = rope(q, k, cos, sin)
    if n_rep > 1:
        k = np.repeat(k, n_rep, axis=2)
        v = np.repeat(v, n_rep, axis=2)
    q = q.transpose(0, 2, 1, 3)
    k = k.transpose(0, 2, 1, 3)
    v = v.transpose(0, 2, 1, 3)
    scores = (q @ k.transpose(0, 1, 3, 2)) / np.sqrt(head_dim)
    causal_mask = np.triu(np.ones((S, S)) * -10000.0, k=1).astype(scores.dtype)
    scores = scores + causal_mask[None, None, :, :]
    attn = softmax(scores) @ v
    attn = attn.transpose(0, 2, 1, 3).reshape(B, S, nq * head_dim)
    o = attn @ o_weight
    if tp_world > 1:
        o = cc.all_reduce(o, replica_groups=[list(range(tp_world))], reduce_op=np.add)
    h1 = x + o
    h2 = rmsnorm(h1, post_norm_weight, eps)
    gate, up = np.split(h2 @ gate_up_weight, 2, axis=-1)
    d = (silu(gate) * up) @ down_weight
    if tp_world > 1:
        d = cc.all_reduce(d, replica_groups=[list(range(tp_world))], reduce_op=np.add)
    return h1 + d


# ---------------------------------------------------------------------------
# elementwise chain and layout move (the memory-bound kernel families of the
# path on their own)
# ---------------------------------------------------------------------------
def silu_mul_kernel(gate, up):
    """The SwiGLU activation of ``examples/models/qwen3_embedding/kernels/
    ffn.py:11-46`` on its own: one fused elementwise chain (negate, exp, add,
    reciprocal, two multiplies) over two inputs."""
    return silu(gate) * up


def transpose_kernel(x):
    """A materialised 2-D transpose (``core/ops/transform.py:55-79``)."""
    return np.transpose(x)


# ---------------------------------------------------------------------------
# 6. Qwen3 attention with a KV cache (prefill and one-token decode)
# ---------------------------------------------------------------------------
def qk_rmsnorm(x, weight, eps):
    """``examples/models/qwen3/kernels/rmsnorm.py:4-21`` (fp32 compute)."""
    original_dtype = x.dtype
    x = x.astype(np.float32)
    weight = weight.astype(np.float32)
    z = np.mean(np.square(x), axis=-1, keepdims=True)
    z = (z + eps).astype(x.dtype)
    return (x / np.sqrt(z) * weight).astype(original_dtype)


def qwen3_rope_cache(head_dim, max_seq_len, base=1000000.0, dtype=bfloat16):
    """cos/sin tables (max_seq_len, head_dim/2) of the Qwen3 example
    (``examples/models/qwen3/kernels/rope.py:4-21``): inverse frequencies in
    float64, positions in float32, cos/sin evaluated in float32, then cast."""
    inv = 1.0 / (base ** (np.arange(0, head_dim, 2)[: head_dim // 2] / head_dim))
    ang = np.outer(np.arange(max_seq_len, dtype=np.float32), inv)
    return np.cos(ang, dtype=np.float32).astype(dtype), np.sin(ang, dtype=np.float32).astype(dtype)


def cached_attention_kernel(
    x, qkv_weight, q_norm_weight, k_norm_weight, cache_k, cache_v, start_pos, o_weight,
    n_heads=4, head_dim=128, n_kv_heads=2, norm_eps=1e-6, rope_base=1000000.0, tp_world=1,
):
    """One attention block of the reference's Qwen3 decode loop
    (``examples/models/qwen3/kernels/attention.py:25-156``): QKV projection,
    q/k RMSNorm, RoPE, KV-cache update (``cache[:, :S] = k`` at prefill,
    ``cache[:, start_pos] = k`` at decode), GQA repeat, causal scores, softmax,
    PV, o-projection (+ all-reduce under TP).  ``start_pos`` is None for the
    prefill, else a (1,) int32 tensor; the caches are mutated in place (the
    traced kernel returns them as aliased outputs).  The rotary and mask
    tables are trace-time constants, as in the reference."""
    from nkipy_b200.core import tensor_apis

    is_prefill = start_pos is None
    B, S, _ = x.shape
    nq = n_heads // tp_world
    nkv = max(1, n_kv_heads // tp_world)
    n_rep = nq // nkv
    s0, s1 = nq * head_dim, (nq + nkv) * head_dim
    xq, xk, xv = np.split(np.matmul(x, qkv_weight), [s0, s1], axis=x.ndim - 1)
    xq = qk_rmsnorm(xq.reshape(B, S, nq, head_dim), q_norm_weight, norm_eps)
    xk = qk_rmsnorm(xk.reshape(B, S, nkv, head_dim), k_norm_weight, norm_eps)
    xv = xv.reshape(B, S, nkv, head_dim)

    L = cache_k.shape[1]
    cos_t, sin_t = qwen3_rope_cache(head_dim, L, rope_base)
    if is_prefill:
        cos, sin = cos_t[0:S], sin_t[0:S]
    else:
        cos = tensor_apis.constant(cos_t)[start_pos]
        sin = tensor_apis.constant(sin_t)[start_pos]
    xq, xk = rope(xq, xk, cos, sin)

    if is_prefill:
        cache_k[:, :S] = xk
        cache_v[:, :S] = xv
    else:
        cache_k[:, start_pos] = xk
        cache_v[:, start_pos] = xv

    keys = np.repeat(cache_k, n_rep, axis=2) if n_rep > 1 else cache_k
    values = np.repeat(cache_v, n_rep, axis=2) if n_rep > 1 else cache_v
    xq = xq.transpose(0, 2, 1, 3)
    keys = keys.transpose(0, 2, 1, 3)
    values = values.transpose(0, 2, 1, 3)
    scores = (xq @ keys.transpose(0, 1, 3, 2)) / np.float32(np.sqrt(head_dim))
    scores = scores.astype(bfloat16)
    mask = np.triu(np.ones((L, L)) * -100000, k=1).astype(scores.dtype)
    mask = tensor_apis.constant(mask)
    if is_prefill:
        scores = scores + np.expand_dims(mask[:S, :L], axis=[0, 1])
    else:
        scores = scores + np.expand_dims(mask[start_pos, :L], axis=[0, 1])
    exp_s = np.exp(scores - np.max(scores, axis=-1, keepdims=True))
    probs = exp_s / np.sum(exp_s, axis=-1, keepdims=True)
    out = (probs @ values).transpose(0, 2, 1, 3).reshape(B, S, -1)
    out = np.matmul(out, o_weight)
    if tp_world > 1:
        out = cc.all_reduce(out, replica_groups=[list(range(tp_world))], reduce_op=np.add)
    return out


def greedy_sampling_kernel(h, norm_weight, lm_head_weight, max_batch_size=1, norm_eps=1e-6, tp_world=1):
    """Greedy next-token choice over a vocabulary split across ranks, as the
    reference's ``greedy_sampling`` (``examples/models/qwen3/kernels/
    sampling.py:113-147``): RMSNorm, last-position logits of this rank's
    vocabulary shard, top-1 per rank, all-gather of the ranks' maxima and ids,
    top-1 over the ranks, global id = rank * shard + local id."""
    from nkipy_b200.core import tensor_apis

    h = qk_rmsnorm(h, norm_weight, norm_eps)
    logits = h[:, -1, :] @ lm_head_weight
    logits, next_id = tensor_apis.topk(logits, k=1, axis=1)
    group = [list(range(tp_world))]
    logits_all = cc.all_gather(logits, all_gather_dim=1, replica_groups=group)
    next_id_all = cc.all_gather(next_id, all_gather_dim=1, replica_groups=group)
    _, top_index = tensor_apis.topk(logits_all, k=1, axis=1)
    final_next_id = np.empty_like(next_id)
    vocab_per_device = lm_head_weight.shape[1]
    for b in range(max_batch_size):
        device_idx = top_index[b]
        local_idx = next_id_all[b, device_idx]
        final_next_id[b] = device_idx * vocab_per_device + local_idx
    return final_next_id


def rope_tables(seq_len, head_dim, theta=500000.0):
    """cos/sin tables (S, head_dim/2), as ``qwen3_embedding/kernels/rope.py:4-31``."""
    inv_freq = 1.0 / (theta ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))
    freqs = np.outer(np.arange(seq_len, dtype=np.float32), inv_freq)
    return np.cos(freqs).astype(np.float32), np.sin(freqs).astype(np.float32)


# ---------------------------------------------------------------------------
# Synthetic inputs
# ---------------------------------------------------------------------------
@dataclass(frozen=True)
class LayerShape:
    batch: int = 4
    seq: int = 2048
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    theta: float = 500000.0
    eps: float = 1e-6


def layer_weights(shape: LayerShape, seed=0):
    """Full (unsharded) bf16 weights ~ N(0, 0.02), used as ``x @ W``."""
    rng = np.random.default_rng(seed)
    hd = shape.head_dim

    def w(r, c):
        return (rng.standard_normal((r, c), dtype=np.float32) * 0.02).astype(bfloat16)

    return {
        "qkv": w(shape.hidden, (shape.n_heads + 2 * shape.n_kv_heads) * hd),
        "o": w(shape.n_heads * hd, shape.hidden),
        "gate": w(shape.hidden, shape.ffn),
        "up": w(shape.hidden, shape.ffn),
        "down": w(shape.ffn, shape.hidden),
        "ln1": np.ones(shape.hidden, dtype=bfloat16),
        "ln2": np.ones(shape.hidden, dtype=bfloat16),
    }


def shard_layer_weights(full, shape: LayerShape, rank, world):
    """Column/row split of one rank (``examples/models/qwen3/tensor_preparation.py:15-31``)."""
    hd = shape.head_dim
    nq, nkv = shape.n_heads // world, max(1, shape.n_kv_heads // world)
    if shape.n_kv_heads % world or shape.n_heads % world:
        raise ValueError(f"tp world {world} must divide the head counts")
    q_cols = slice(rank * nq * hd, (rank + 1) * nq * hd)
    k0 = shape.n_heads * hd
    v0 = k0 + shape.n_kv_heads * hd
    # local q head i of this rank reads local kv head i // (nq // nkv)
    kv_cols = slice(rank * nkv * hd, (rank + 1) * nkv * hd)
    qkv = np.concatenate(
        [
            full["qkv"][:, q_cols],
            full["qkv"][:, k0 + kv_cols.start : k0 + kv_cols.stop],
            full["qkv"][:, v0 + kv_cols.start : v0 + kv_cols.stop],
        ],
        axis=1,
    )
    f = shape.ffn // world
    fs = slice(rank * f, (rank + 1) * f)
    gate_up = np.concatenate([full["gate"][:, fs], full["up"][:, fs]], axis=1)
    return {
        "qkv": np.ascontiguousarray(qkv),
        "o": np.ascontiguousarray(full["o"][q_cols, :]),
        "gate_up": np.ascontiguousarray(gate_up),
        "down": np.ascontiguousarray(full["down"][fs, :]),
        "ln1": full["ln1"],
        "ln2": full["ln2"],
    }


def layer_args(x, shard, shape: LayerShape, world):
    # bf16 tables, as the reference's TP attention builds them
    # (examples/models/qwen3/kernels/attention.py: compute_cos_sin_cache(..., dtype=bfloat16))
    cos, sin = (t.astype(x.dtype) for t in rope_tables(x.shape[1], shape.head_dim, shape.theta))
    args = (x, shard["ln1"], shard["qkv"], shard["o"], shard["ln2"], shard["gate_up"], shard["down"], cos, sin)
    kwargs = dict(
        n_heads=shape.n_heads, n_kv_heads=shape.n_kv_heads, head_dim=shape.head_dim, eps=shape.eps, tp_world=world
    )
    return args, kwargs


def make_inputs(config, seed=0, scale=1.0):
    """Seeded inputs of a configuration; ``scale`` < 1 shrinks the leading dim."""
    rng = np.random.default_rng(seed)
    if config == "softmax":
        rows = max(1, int(4096 * scale))
        return (rng.standard_normal((rows, 4096), dtype=np.float32),)
    if config == "rmsnorm":
        rows = max(1, int(16384 * scale))
        x = rng.standard_normal((rows, 4096), dtype=np.float32)
        r = rng.standard_normal((rows, 4096), dtype=np.float32)
        w = rng.uniform(0.5, 1.5, 4096).astype(np.float32)
        return (x, r, w)
    if config == "gemm":
        n = max(64, int(8192 * scale))
        a = (rng.standard_normal((n, 8192), dtype=np.float32) * 0.02).astype(bfloat16)
        b = (rng.standard_normal((8192, 8192), dtype=np.float32) * 0.02).astype(bfloat16)
        return (a, b)
    if config == "bmm":
        bsz = max(1, int(32 * scale))
        a = (rng.standard_normal((bsz, 2048, 2048), dtype=np.float32) * 0.02).astype(bfloat16)
        b = (rng.standard_normal((bsz, 2048, 2048), dtype=np.float32) * 0.02).astype(bfloat16)
        return (a, b)
    if config == "linattn":
        bsz = max(1, int(8 * scale))
        shp = (bsz, 16, 4096, 128)
        return tuple(rng.standard_normal(shp, dtype=np.float32).astype(bfloat16) for _ in range(3))
    raise ValueError(f"unknown config {config}")


KERNELS = {
    "softmax": softmax_kernel,
    "rmsnorm": residual_rmsnorm_kernel,
    "gemm": matmul_kernel,
    "bmm": bmm_kernel,
    "linattn": chunked_linear_attention_kernel,
    "layer": llama_decoder_layer_kernel,
}
