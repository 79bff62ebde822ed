"""Rotary embedding, causal attention with grouped KV heads, a decoder block."""

import ml_dtypes
import numpy as np

from nkipy_b200.core.specs import KernelSpec, ShapeSpec, TensorInputSpec, TypeSpec

_BF = TypeSpec(allowed=[np.dtype(ml_dtypes.bfloat16)], default=np.dtype(ml_dtypes.bfloat16))
_F32 = TypeSpec(allowed=[np.float32], default=np.float32)


def rotary(x, cos, sin):
    """Half-split rotation of (batch, seq, heads, dim) by (seq, dim / 2) tables."""
    half = x.shape[-1] // 2
    c = cos[None, :, None, :]
    s = sin[None, :, None, :]
    x0, x1 = x[..., :half], x[..., half:]
    return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)


def causal_gqa_attention(q, k, v):
    """q (B, S, H, D), k / v (B, S, Hkv, D); H a multiple of Hkv."""
    rep = q.shape[2] // k.shape[2]
    k = np.repeat(k, rep, axis=2)
    v = np.repeat(v, rep, axis=2)
    q, k, v = q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3)
    s = (q @ k.transpose(0, 1, 3, 2)) / np.sqrt(q.shape[-1])
    n = q.shape[2]
    s = s + np.triu(np.ones((n, n)) * -10000.0, k=1).astype(s.dtype)
    x = s.astype(np.float32)
    e = np.exp(x - np.max(x, axis=-1, keepdims=True))
    p = (e / np.sum(e, axis=-1, keepdims=True)).astype(s.dtype)
    return (p @ v).transpose(0, 2, 1, 3)


def decoder_block_fp32(x, wq, wk, wv, wo, w1, w2, g1, g2):
    """Pre-norm block: RMSNorm, single-head causal attention, RMSNorm, ReLU MLP."""

    def norm(t, g):
        return t / np.sqrt(np.mean(t * t, axis=-1, keepdims=True) + 1e-6) * g

    h = norm(x, g1)
    q, k, v = h @ wq, h @ wk, h @ wv
    s = (q @ k.T) / np.sqrt(q.shape[-1])
    n = x.shape[0]
    s = s + np.triu(np.ones((n, n), dtype=np.float32) * -1e9, k=1)
    e = np.exp(s - np.max(s, axis=-1, keepdims=True))
    a = (e / np.sum(e, axis=-1, keepdims=True)) @ v
    x = x + a @ wo
    return x + np.maximum(norm(x, g2) @ w1, 0.0) @ w2


def _t(dt, dims, default, value=None):
    return TensorInputSpec(dtype_spec=dt, shape_spec=ShapeSpec(dims, default), default_value=value)


_COS, _SIN = (f(np.outer(np.arange(64), 1.0 / 10000 ** (np.arange(0, 64, 2) / 64))).astype(np.float32)
              for f in (np.cos, np.sin))
kernel_specs = [
    KernelSpec(rotary, [_t(_F32, [2, 64, 4, 64], (2, 64, 4, 64)), _t(_F32, [64, 32], (64, 32), _COS),
                        _t(_F32, [64, 32], (64, 32), _SIN)], description="rotary embedding"),
    KernelSpec(causal_gqa_attention, [_t(_BF, [(1, 4), (1, 512), 8, 128], (2, 256, 8, 128)),
                                      _t(_BF, [(1, 4), (1, 512), 2, 128], (2, 256, 2, 128)),
                                      _t(_BF, [(1, 4), (1, 512), 2, 128], (2, 256, 2, 128))],
               description="causal attention, 4 query heads per KV head, head_dim 128 (tensor-core flash kernel)"),
    KernelSpec(causal_gqa_attention, [_t(_BF, [1, 96, 4, 64], (1, 96, 4, 64)), _t(_BF, [1, 96, 4, 64], (1, 96, 4, 64)),
                                      _t(_BF, [1, 96, 4, 64], (1, 96, 4, 64))],
               description="causal attention, head_dim 64"),
    KernelSpec(decoder_block_fp32, [_t(_F32, [(2, 128), 32], (40, 32))] + [_t(_F32, [32, 32], (32, 32))] * 4 +
               [_t(_F32, [32, 64], (32, 64)), _t(_F32, [64, 32], (64, 32)), _t(_F32, [32], (32,)),
                _t(_F32, [32], (32,))], description="small fp32 pre-norm decoder block"),
]
