"""KV-cache decode on the device: in-place updates of mutated parameters.

Follows the reference's Qwen3 decode loop (``examples/models/qwen3/qwen3.py:280-336``):
a prefill kernel and a one-token decode kernel are compiled once, the caches
stay resident as device tensors bound both as ``cache_k.must_alias_input``
and ``cache_k``, and every step's output and the caches are compared with the
NumPy direct call of the same kernel body.
"""

import contextlib

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200 import workloads as W
from nkipy_b200.runtime import DeviceKernel, DeviceTensor
from oracle import numpy_ref as O
from tests.utils import BF16_RTOL, assert_close, on_device, sum_abs_atol

BF16 = np.dtype(ml_dtypes.bfloat16)
pytestmark = pytest.mark.gpu


def _inputs(B, L, nq, nkv, hd, D, S, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, S, D), dtype=np.float32).astype(BF16)
    wqkv = (rng.standard_normal((D, (nq + 2 * nkv) * hd), dtype=np.float32) * 0.02).astype(BF16)
    wo = (rng.standard_normal((nq * hd, D), dtype=np.float32) * 0.02).astype(BF16)
    qn = rng.uniform(0.5, 1.5, hd).astype(BF16)
    kn = rng.uniform(0.5, 1.5, hd).astype(BF16)
    return x, wqkv, qn, kn, wo


@pytest.mark.parametrize("B,L,nq,nkv,hd,D,S,steps", [(2, 128, 8, 2, 128, 1024, 32, 4), (1, 64, 4, 4, 64, 256, 8, 3)])
def test_kv_cache_prefill_then_decode(B, L, nq, nkv, hd, D, S, steps):
    kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
    x, wqkv, qn, kn, wo = _inputs(B, L, nq, nkv, hd, D, S)
    rng = np.random.default_rng(1)
    tokens = [rng.standard_normal((B, 1, D), dtype=np.float32).astype(BF16) for _ in range(steps)]

    # NumPy direct call (the reference's CPU mode): caches mutated in place
    ck = np.zeros((B, L, nkv, hd), BF16)
    cv = np.zeros((B, L, nkv, hd), BF16)
    want = [W.cached_attention_kernel(x, wqkv, qn, kn, ck, cv, None, wo, **kw)]
    for i, t in enumerate(tokens):
        want.append(W.cached_attention_kernel(t, wqkv, qn, kn, ck, cv, np.array([S + i], np.int32), wo, **kw))

    zeros = np.zeros((B, L, nkv, hd), BF16)
    pre = DeviceKernel.compile_and_load(W.cached_attention_kernel, x, wqkv, qn, kn, zeros, zeros, None, wo,
                                        name="cache_prefill", **kw)
    dec = DeviceKernel.compile_and_load(W.cached_attention_kernel, tokens[0], wqkv, qn, kn, zeros, zeros,
                                        np.array([S], np.int32), wo, name="cache_decode", **kw)
    dk, dv = DeviceTensor.from_numpy(zeros), DeviceTensor.from_numpy(zeros)
    w = {n: DeviceTensor.from_numpy(a) for n, a in
         (("qkv_weight", wqkv), ("q_norm_weight", qn), ("k_norm_weight", kn), ("o_weight", wo))}
    out = DeviceTensor.empty((B, S, D), BF16)
    pre(inputs=dict(w, x=DeviceTensor.from_numpy(x), **{"cache_k.must_alias_input": dk, "cache_v.must_alias_input": dv}),
        outputs={"output0": out, "cache_k": dk, "cache_v": dv})
    got = [out.numpy()]
    out1 = DeviceTensor.empty((B, 1, D), BF16)
    for i, t in enumerate(tokens):
        dec(inputs=dict(w, x=DeviceTensor.from_numpy(t), start_pos=DeviceTensor.from_numpy(np.array([S + i], np.int32)),
                        **{"cache_k.must_alias_input": dk, "cache_v.must_alias_input": dv}),
            outputs={"output0": out1, "cache_k": dk, "cache_v": dv})
        got.append(out1.numpy())
    for g, e in zip(got, want):
        assert_close(g, e, BF16_RTOL)
    assert_close(dk.numpy(), ck, BF16_RTOL)
    assert_close(dv.numpy(), cv, BF16_RTOL)


def test_mutated_parameter_keeps_old_value_for_earlier_readers():
    """A value read from a parameter before the kernel overwrites part of it
    must see the old contents, also when the caller binds the output in place."""

    def k(a, idx, v):
        old = a * 2.0
        a[:, idx] = v
        return old + a

    rng = np.random.default_rng(2)
    a = rng.standard_normal((6, 10, 5), dtype=np.float32)
    idx = np.array([7], np.int32)
    v = rng.standard_normal((6, 1, 5), dtype=np.float32)
    a_cpu = a.copy()
    want = k(a_cpu, idx, v)
    a_dev = a.copy()
    got = on_device(k, a_dev, idx, v)  # the one-shot path binds the mutated input in place
    assert_close(got, want, 1e-6)
    np.testing.assert_array_equal(a_dev, a_cpu)


def test_successive_updates_in_place():
    def k(a, i, j, v, w):
        a[i] = v
        a[j] = w
        a[0:2] = 0.0
        return a.sum(axis=1)

    rng = np.random.default_rng(3)
    a = rng.standard_normal((9, 33), dtype=np.float32)
    i, j = np.array([4], np.int32), np.array([7], np.int32)
    v = rng.standard_normal((1, 33), dtype=np.float32)
    w = rng.standard_normal((1, 33), dtype=np.float32)
    a_cpu, a_dev = a.copy(), a.copy()
    want = k(a_cpu, i, j, v, w)
    got = on_device(k, a_dev, i, j, v, w)
    assert_close(got, want, 1e-5, atol=sum_abs_atol(a_cpu, axis=1))
    np.testing.assert_array_equal(a_dev, a_cpu)


@pytest.mark.parametrize("B,L,nq,nkv", [(2, 320, 16, 2), (3, 200, 8, 8), (2, 320, 8, 4), (1, 200, 16, 4)])
def test_decode_attention_at_cache_edges(B, L, nq, nkv):
    """The fused decode attention over random caches at the first position,
    interior positions and the last row of the cache; several key chunks per
    KV head and 1 to 8 query heads per KV head.  Up to 64 keys the plain direct
    call is the reference; beyond, its bf16 softmax sum (accumulated in order
    in bf16) stagnates, so the direct call with that sum accumulated in fp32
    is (the rest of the body unchanged)."""
    hd, D = 128, 512
    kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
    x, wqkv, qn, kn, wo = _inputs(B, L, nq, nkv, hd, D, 1, seed=5)
    rng = np.random.default_rng(6)
    ck0 = rng.standard_normal((B, L, nkv, hd), dtype=np.float32).astype(BF16)
    cv0 = rng.standard_normal((B, L, nkv, hd), dtype=np.float32).astype(BF16)
    dec = DeviceKernel.compile_and_load(W.cached_attention_kernel, x, wqkv, qn, kn, ck0, cv0,
                                        np.array([0], np.int32), wo, name="cache_decode_edges", **kw)
    w = {n: DeviceTensor.from_numpy(a) for n, a in
         (("qkv_weight", wqkv), ("q_norm_weight", qn), ("k_norm_weight", kn), ("o_weight", wo))}
    xd = DeviceTensor.from_numpy(x)
    for pos in (0, 1, 63, 64, L // 2 + 7, L - 1):
        ck, cv = ck0.copy(), cv0.copy()
        with contextlib.nullcontext() if pos <= 64 else O.fp32_accumulated_bf16_sums():
            want = W.cached_attention_kernel(x, wqkv, qn, kn, ck, cv, np.array([pos], np.int32), wo, **kw)
        dk, dv = DeviceTensor.from_numpy(ck0), DeviceTensor.from_numpy(cv0)
        out = DeviceTensor.empty((B, 1, D), BF16)
        dec(inputs=dict(w, x=xd, start_pos=DeviceTensor.from_numpy(np.array([pos], np.int32)),
                        **{"cache_k.must_alias_input": dk, "cache_v.must_alias_input": dv}),
            outputs={"output0": out, "cache_k": dk, "cache_v": dv})
        assert_close(out.numpy(), want, BF16_RTOL)
        for got, exp in ((dk.numpy(), ck), (dv.numpy(), cv)):
            # the new token's row is computed (bf16 rounding of a different
            # accumulation order); every other row is untouched, bit for bit
            assert_close(got[:, pos], exp[:, pos], BF16_RTOL)
            keep = np.arange(L) != pos
            np.testing.assert_array_equal(got[:, keep].view(np.uint16), exp[:, keep].view(np.uint16))
