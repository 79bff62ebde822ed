"""The CPU oracle reproduces the reference's own NumPy kernel bodies.

Golden vectors were produced by running the reference's functions
(tests/kernels/softmax.py, examples/models/qwen3_embedding/kernels/*,
core/ops/collectives.py cpu implementations) -- see tests/golden/make_golden.py.
"""

import os

import ml_dtypes
import pytest
import numpy as np

from nkipy_b200 import workloads as W
from oracle import numpy_ref as O

BF16 = np.dtype(ml_dtypes.bfloat16)
_z = np.load(os.path.join(os.path.dirname(__file__), "golden", "vectors.npz"))
_bf = set(_z["_bf16_keys"].tolist())


def V(k):
    a = _z[k]
    return a.view(BF16) if k in _bf else a


def test_softmax_vectors():
    for i in range(3):
        np.testing.assert_allclose(O.softmax(V(f"softmax{i}_x")), V(f"softmax{i}_y"), rtol=1e-6, atol=1e-7)
        # the workload body traced by the bench is the same computation
        np.testing.assert_allclose(W.softmax_kernel(V(f"softmax{i}_x")), V(f"softmax{i}_y"), rtol=1e-6, atol=1e-7)


def test_rmsnorm_vectors():
    got = O.residual_rmsnorm(V("rms_x"), V("rms_r"), V("rms_w"), 1e-6)
    np.testing.assert_allclose(got, V("rms_y"), rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(W.residual_rmsnorm_kernel(V("rms_x"), V("rms_r"), V("rms_w")), V("rms_y"), rtol=1e-6, atol=1e-6)


def test_rope_vectors():
    cos, sin = O.rope_tables(64, 128, 500000.0)
    np.testing.assert_allclose(cos, V("rope_cos"), rtol=1e-6)
    np.testing.assert_allclose(sin, V("rope_sin"), rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(O._rope(V("rope_q"), cos, sin), V("rope_qo"), rtol=1e-5, atol=1e-6)
    q, k = W.rope(V("rope_q"), V("rope_k"), cos, sin)
    np.testing.assert_allclose(q, V("rope_qo"), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(k, V("rope_ko"), rtol=1e-5, atol=1e-6)


def test_layer_vectors():
    w = {
        "qkv": V("layer_qkv"), "o": V("layer_o"), "gate": V("layer_gate"), "up": V("layer_up"), "down": V("layer_down"),
        "ln1": np.ones(256, BF16), "ln2": np.ones(256, BF16),
    }
    got = O.llama_layer(V("layer_x"), w, n_heads=4, n_kv_heads=2, head_dim=64, eps=1e-6, theta=500000.0)
    want = V("layer_y")
    err = np.max(np.abs(got.astype(np.float32) - want)) / np.max(np.abs(want))
    assert err < 2e-2, err
    # the traced workload body (TP=1) computes the same layer
    s = W.LayerShape(batch=1, seq=32, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512)
    shard = W.shard_layer_weights(w, s, 0, 1)
    args, kw = W.layer_args(V("layer_x"), shard, s, 1)
    y2 = W.llama_decoder_layer_kernel(*args, **kw)
    err2 = np.max(np.abs(np.asarray(y2, np.float32) - want)) / np.max(np.abs(want))
    assert err2 < 2e-2, err2


def test_collective_cpu_semantics():
    from nkipy_b200.core.ops import collectives as C

    d = V("cc_in")
    np.testing.assert_array_equal(C.all_reduce(d, replica_groups=[[0, 1, 2, 3]]), V("cc_all_reduce_w4"))
    np.testing.assert_array_equal(C.all_gather(d, all_gather_dim=1, replica_groups=[[0, 1]]), V("cc_all_gather_w2"))
    np.testing.assert_array_equal(
        C.reduce_scatter(d, reduce_scatter_dim=0, replica_groups=[[0, 1]]), V("cc_reduce_scatter_w2")
    )
    np.testing.assert_array_equal(
        C.all_to_all(d, split_dimension=1, concat_dimension=0, replica_groups=[[0, 1]]), V("cc_all_to_all_w2")
    )
    np.testing.assert_array_equal(O.all_reduce_identical(d, 4), V("cc_all_reduce_w4"))
    np.testing.assert_array_equal(C.all_gather(d, all_gather_dim=0, replica_groups=[[0, 1]]), V("cc_all_gather_w2_d0"))
    np.testing.assert_array_equal(O.all_gather_identical(d, 2, 0), V("cc_all_gather_w2_d0"))
    np.testing.assert_array_equal(O.all_gather_identical(d, 2, 1), V("cc_all_gather_w2"))
    np.testing.assert_array_equal(
        C.reduce_scatter(d, reduce_scatter_dim=1, replica_groups=[[0, 1]]), V("cc_reduce_scatter_w2_d1")
    )
    np.testing.assert_array_equal(O.reduce_scatter_identical(d, 2, 1), V("cc_reduce_scatter_w2_d1"))
    np.testing.assert_array_equal(O.reduce_scatter_identical(d, 2, 0), V("cc_reduce_scatter_w2"))
    np.testing.assert_array_equal(
        C.all_to_all(d, split_dimension=1, concat_dimension=1, replica_groups=[[0, 1]]), V("cc_all_to_all_w2_d1")
    )


@pytest.mark.parametrize("k", [1, 5, 17])
@pytest.mark.parametrize("asc", [False, True])
def test_topk_vectors(k, asc):
    """The oracle's top-k equals the reference CPU top-k on distinct values."""
    from nkipy_b200.core.ops import nn as NN

    x = V("topk_x")
    vals, ids = O.topk(x, k, is_ascend=asc)
    np.testing.assert_array_equal(vals, V(f"topk_k{k}_a{int(asc)}_v"))
    np.testing.assert_array_equal(ids, V(f"topk_k{k}_a{int(asc)}_i"))
    v2, i2 = NN.topk(x, k, axis=-1, is_ascend=asc)  # this package's CPU op
    np.testing.assert_array_equal(i2, ids)


def test_qwen3_cached_attention_vectors():
    """The cached-attention kernel body reproduces the reference's Qwen3
    attention kernel, prefill then two decode steps on one KV cache."""
    B, L, nq, nkv, hd, D, S = 2, 16, 4, 2, 64, 256, 8
    kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
    args = [V("qa_wqkv"), V("qa_qn"), V("qa_kn")]
    ck = np.zeros((B, L, nkv, hd), W.bfloat16)
    cv = np.zeros((B, L, nkv, hd), W.bfloat16)
    y0 = W.cached_attention_kernel(V("qa_x"), *args, ck, cv, None, V("qa_wo"), **kw)
    np.testing.assert_array_equal(np.asarray(y0, np.float32), V("qa_y0"))
    for i in range(2):
        y = W.cached_attention_kernel(V(f"qa_t{i + 1}"), *args, ck, cv, np.array([S + i], np.int32), V("qa_wo"), **kw)
        np.testing.assert_array_equal(np.asarray(y, np.float32), V(f"qa_y{i + 1}"))
    np.testing.assert_array_equal(ck.view(np.uint16), V("qa_cache_k").view(np.uint16))
    np.testing.assert_array_equal(cv.view(np.uint16), V("qa_cache_v").view(np.uint16))


def test_linear_attention_forms_agree():
    rng = np.random.default_rng(3)
    q, k, v = (rng.standard_normal((1, 2, 256, 32), dtype=np.float32) for _ in range(3))
    a = W.chunked_linear_attention_kernel(q, k, v, chunk=64)
    b = O.linear_attention_recurrent(q, k, v, chunk=64)
    np.testing.assert_allclose(a, b, rtol=2e-4, atol=1e-5)
    # chunk size does not change the result (pure reassociation)
    c = O.linear_attention_recurrent(q, k, v, chunk=16)
    np.testing.assert_allclose(b, c, rtol=2e-4, atol=1e-5)


def test_convolution_vectors():
    """The oracle's convolution and this package's CPU conv ops equal the
    reference's CPU conv2d / conv3d (core/ops/conv.py)."""
    from nkipy_b200.core.ops import conv as CV

    y2 = O.conv_nd(V("conv2_x"), V("conv2_w"), V("conv2_b"), stride=(2, 1), padding=(1, 2))
    np.testing.assert_allclose(y2, V("conv2_y"), rtol=1e-5, atol=1e-5)
    y3 = O.conv_nd(V("conv3_x"), V("conv3_w"), None, stride=(1, 2, 1), padding=1)
    np.testing.assert_allclose(y3, V("conv3_y"), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(CV.conv2d(V("conv2_x"), V("conv2_w"), V("conv2_b"), stride=(2, 1), padding=(1, 2)),
                               V("conv2_y"), rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(CV.conv3d(V("conv3_x"), V("conv3_w"), None, stride=(1, 2, 1), padding=1), V("conv3_y"),
                               rtol=1e-6, atol=1e-6)


def test_bf16_sum_accumulation_modes():
    """NumPy sums ml_dtypes bf16 in order with bf16 rounding (stagnates);
    the fp32-accumulated mode rounds once and leaves np.sum as it found it."""
    a = np.full(1000, 0.2, O.bfloat16)
    assert float(np.sum(a)) == 64.0
    plain = np.sum
    with O.fp32_accumulated_bf16_sums():
        assert float(np.sum(a)) == 200.0
        assert np.sum(a.reshape(10, 100), axis=-1, keepdims=True).shape == (10, 1)
        assert np.sum(np.ones(5, np.float32)).dtype == np.float32
    assert np.sum is plain
