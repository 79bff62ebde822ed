"""Generate the golden fixtures of this folder from the reference itself.

Run in an environment where the reference tree (shaojiex-aws/nkipy) is
available (``NKIPY_REFERENCE_ROOT``):

    python tests/golden/make_golden.py

Writes:
  oplists.json    the reference tracer's graph (ops, shapes, dtypes,
                  attributes, result names, aliases) for golden_kernels.CASES
  promotion.json  the reference promotion table over all pairs of type keys
  vectors.npz     outputs of the reference's own NumPy kernel bodies
                  (tests/kernels/softmax.py; examples/models/qwen3_embedding
                  kernels rmsnorm, softmax, rope, ffn; a Llama layer composed
                  from them; the Qwen3 attention kernel with its KV cache,
                  prefill and decode), of its CPU collective semantics and
                  of its CPU top-k, on seeded inputs
The tests only read these files.
"""

import importlib.util
import json
import os
import sys

import ml_dtypes
import numpy as np
import torch.distributed  # noqa: F401  (before the protobuf stubs, which confuse torch's import-time inspection)

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from refimport import REF_ROOT, import_reference  # noqa: E402

BF16 = np.dtype(ml_dtypes.bfloat16)


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, os.path.join(REF_ROOT, path))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def oplists():
    import golden_kernels as G

    ref_trace, _ = import_reference()
    import nkipy.core.ops as ref_ops

    G.OPS = ref_ops
    out = {}
    for name, fn, make, kw in G.CASES:
        k = ref_trace.NKIPyKernel.trace(fn, backend="hlo")
        g = k.specialize(*make(), **kw)
        out[name] = G.describe(g)
    return out


def promotion():
    _, hlo = import_reference()
    keys = {
        "bool": np.bool_,
        "weak_int": hlo._WeakInt,
        "weak_float": hlo._WeakFloat,
        "int8": np.int8,
        "int16": np.int16,
        "int32": np.int32,
        "int64": np.int64,
        "uint8": np.uint8,
        "uint16": np.uint16,
        "uint32": np.uint32,
        "uint64": np.uint64,
        "float16": np.float16,
        "float32": np.float32,
        "float64": np.float64,
        "bfloat16": ml_dtypes.bfloat16,
        "float8_e5m2": ml_dtypes.float8_e5m2,
        "float8_e4m3fn": ml_dtypes.float8_e4m3fn,
        "float8_e4m3": ml_dtypes.float8_e4m3,
    }
    table = {}
    for a, ka in keys.items():
        for b, kb in keys.items():
            try:
                r = hlo._lookup_promotion(ka, kb)
                table[f"{a},{b}"] = None if r is None else np.dtype(r).name
            except TypeError:
                table[f"{a},{b}"] = "TypeError"
    return table


def vectors():
    import_reference()
    rng = np.random.default_rng(2024)
    v = {}
    sm = _load("tests/kernels/softmax.py", "ref_softmax")
    for i, shape in enumerate([(8, 128), (7, 1000), (3, 4096)]):
        x = rng.standard_normal(shape, dtype=np.float32)
        v[f"softmax{i}_x"] = x
        v[f"softmax{i}_y"] = sm.softmax_kernel(x)

    qe = os.path.join(REF_ROOT, "examples", "models", "qwen3_embedding")
    sys.path.insert(0, qe)
    rms = _load("examples/models/qwen3_embedding/kernels/rmsnorm.py", "ref_rms")
    smx = _load("examples/models/qwen3_embedding/kernels/softmax.py", "ref_smx")
    rope = _load("examples/models/qwen3_embedding/kernels/rope.py", "ref_rope")
    ffn = _load("examples/models/qwen3_embedding/kernels/ffn.py", "ref_ffn")

    x = rng.standard_normal((16, 512), dtype=np.float32)
    r = rng.standard_normal((16, 512), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, 512).astype(np.float32)
    v["rms_x"], v["rms_r"], v["rms_w"] = x, r, w
    v["rms_y"] = rms.rmsnorm(x + r, w, 1e-6)

    cos, sin = rope.compute_qwen3_cos_sin(64, 128, theta=500000.0)
    v["rope_cos"], v["rope_sin"] = cos, sin
    q = rng.standard_normal((2, 64, 4, 128), dtype=np.float32)
    k = rng.standard_normal((2, 64, 2, 128), dtype=np.float32)
    qo, ko = rope.rope_qwen3(q, k, cos, sin)
    v["rope_q"], v["rope_k"], v["rope_qo"], v["rope_ko"] = q, k, qo, ko

    # small Llama layer composed from the reference's own pieces (bf16)
    B, S, H, nq, nkv, hd, F = 1, 32, 256, 4, 2, 64, 512
    wr = lambda r_, c_: (rng.standard_normal((r_, c_), dtype=np.float32) * 0.02).astype(BF16)  # noqa: E731
    Wqkv, Wo, Wg, Wu, Wd = wr(H, (nq + 2 * nkv) * hd), wr(nq * hd, H), wr(H, F), wr(H, F), wr(F, H)
    ln1 = np.ones(H, BF16)
    ln2 = np.ones(H, BF16)
    xl = rng.standard_normal((B, S, H), dtype=np.float32).astype(BF16)
    c2, s2 = rope.compute_qwen3_cos_sin(S, hd, theta=500000.0)
    h = rms.rmsnorm(xl, ln1, 1e-6)
    qkv = h @ Wqkv
    qq, kk, vv = np.split(qkv, [nq * hd, (nq + nkv) * hd], axis=-1)
    qq = qq.reshape(B, S, nq, hd)
    kk = kk.reshape(B, S, nkv, hd)
    vv = vv.reshape(B, S, nkv, hd)
    qq, kk = rope.rope_qwen3(qq, kk, c2, s2)
    kk = np.repeat(kk, nq // nkv, axis=2)
    vv = np.repeat(vv, nq // nkv, axis=2)
    qq, kk, vv = qq.transpose(0, 2, 1, 3), kk.transpose(0, 2, 1, 3), vv.transpose(0, 2, 1, 3)
    scores = ((qq @ kk.transpose(0, 1, 3, 2)) / np.sqrt(hd)).astype(BF16)
    mask = np.triu(np.ones((S, S)) * -10000.0, k=1).astype(BF16)
    p = smx.softmax(scores + mask[None, None])
    att = (p @ vv).astype(BF16).transpose(0, 2, 1, 3).reshape(B, S, nq * hd)
    h1 = ((att @ Wo) + xl).astype(BF16)
    h2 = rms.rmsnorm(h1, ln2, 1e-6)
    y = ffn.feedforward_kernel(h2, np.concatenate([Wg, Wu], axis=1), Wd) + h1
    v.update(layer_x=xl, layer_qkv=Wqkv, layer_o=Wo, layer_gate=Wg, layer_up=Wu, layer_down=Wd, layer_y=np.asarray(y, np.float32))

    # CPU collective semantics (reference core/ops/collectives.py:17-214)
    from nkipy.core.ops import collectives as C

    d = rng.standard_normal((4, 6), dtype=np.float32)
    v["cc_in"] = d
    v["cc_all_reduce_w4"] = C.all_reduce(d, replica_groups=[[0, 1, 2, 3]])
    v["cc_all_gather_w2"] = C.all_gather(d, all_gather_dim=1, replica_groups=[[0, 1]])
    v["cc_reduce_scatter_w2"] = C.reduce_scatter(d, reduce_scatter_dim=0, replica_groups=[[0, 1]])
    v["cc_all_to_all_w2"] = C.all_to_all(d, split_dimension=1, concat_dimension=0, replica_groups=[[0, 1]])
    v["cc_all_gather_w2_d0"] = C.all_gather(d, all_gather_dim=0, replica_groups=[[0, 1]])
    v["cc_reduce_scatter_w2_d1"] = C.reduce_scatter(d, reduce_scatter_dim=1, replica_groups=[[0, 1]])
    v["cc_all_to_all_w2_d1"] = C.all_to_all(d, split_dimension=1, concat_dimension=1, replica_groups=[[0, 1]])

    # top-k (reference core/ops/nn.py:22-62, CPU implementation) on distinct values
    from nkipy.core.ops import nn as NN

    tx = (rng.permutation(6 * 300).reshape(6, 300).astype(np.float32) - 900.0) / 7.0
    v["topk_x"] = tx
    for kk in (1, 5, 17):
        for asc in (False, True):
            vals, ids = NN.topk(tx, kk, axis=-1, is_ascend=asc)
            v[f"topk_k{kk}_a{int(asc)}_v"], v[f"topk_k{kk}_a{int(asc)}_i"] = vals, ids

    # convolutions (reference core/ops/conv.py CPU implementations)
    from nkipy.core.ops import conv as CV

    cx = rng.standard_normal((2, 3, 9, 11), dtype=np.float32)
    cw = rng.standard_normal((4, 3, 3, 2), dtype=np.float32)
    cb = rng.standard_normal((4,), dtype=np.float32)
    v.update(conv2_x=cx, conv2_w=cw, conv2_b=cb, conv2_y=CV.conv2d(cx, cw, cb, stride=(2, 1), padding=(1, 2)))
    cx3 = rng.standard_normal((1, 2, 5, 6, 7), dtype=np.float32)
    cw3 = rng.standard_normal((3, 2, 2, 3, 2), dtype=np.float32)
    v.update(conv3_x=cx3, conv3_w=cw3, conv3_y=CV.conv3d(cx3, cw3, None, stride=(1, 2, 1), padding=1))

    v.update(qwen3_cached_attention(rng))
    return {k: (a.view(np.uint16) if a.dtype == BF16 else a) for k, a in v.items()}, [k for k, a in v.items() if a.dtype == BF16]


def qwen3_cached_attention(rng):
    """The reference's Qwen3 attention kernel (examples/models/qwen3/kernels/
    attention.py:25-156) called directly on NumPy arrays: a prefill of 8 tokens
    then two one-token decode steps on the same KV cache, world size 1.  Its
    imports of neuronxcc (nki.language.bfloat16, nki.typing) are stubbed with
    ml_dtypes' bfloat16 and placeholders; torch.distributed reports world 1."""
    import types

    for name in ("neuronxcc", "neuronxcc.nki"):
        sys.modules.setdefault(name, types.ModuleType(name))
    lang = types.ModuleType("neuronxcc.nki.language")
    lang.bfloat16 = BF16
    typ = types.ModuleType("neuronxcc.nki.typing")
    typ.tensor = typ.mutable_tensor = typ.mutable = typ.immutable = object
    sys.modules["neuronxcc.nki.language"] = lang
    sys.modules["neuronxcc.nki.typing"] = typ
    sys.path.insert(0, os.path.join(REF_ROOT, "examples", "models", "qwen3"))
    from kernels import attention as A

    A.dist.get_world_size = lambda *a, **k: 1
    B, L, nq, nkv, hd, D, S = 2, 16, 4, 2, 64, 256, 8
    x = rng.standard_normal((B, S, D), dtype=np.float32).astype(BF16)
    wqkv = (rng.standard_normal((D, (nq + 2 * nkv) * hd), dtype=np.float32) * 0.05).astype(BF16)
    wo = (rng.standard_normal((nq * hd, D), dtype=np.float32) * 0.05).astype(BF16)
    qn = rng.uniform(0.5, 1.5, hd).astype(BF16)
    kn = rng.uniform(0.5, 1.5, hd).astype(BF16)
    ck = np.zeros((B, L, nkv, hd), BF16)
    cv = np.zeros((B, L, nkv, hd), BF16)
    v = dict(qa_x=x, qa_wqkv=wqkv, qa_wo=wo, qa_qn=qn, qa_kn=kn)
    v["qa_y0"] = A.attention_kernel(x, wqkv, qn, kn, 1e-6, nq, hd, nkv, ck, cv, None, wo)
    for i in range(2):
        t = rng.standard_normal((B, 1, D), dtype=np.float32).astype(BF16)
        v[f"qa_t{i + 1}"] = t
        v[f"qa_y{i + 1}"] = A.attention_kernel(t, wqkv, qn, kn, 1e-6, nq, hd, nkv, ck, cv,
                                               np.array([S + i], np.int32), wo)
    v["qa_cache_k"], v["qa_cache_v"] = ck.copy(), cv.copy()
    return v


def main():
    with open(os.path.join(HERE, "oplists.json"), "w") as f:
        json.dump(oplists(), f, indent=0, sort_keys=True)
    with open(os.path.join(HERE, "promotion.json"), "w") as f:
        json.dump(promotion(), f, indent=0, sort_keys=True)
    vec, bf = vectors()
    np.savez_compressed(os.path.join(HERE, "vectors.npz"), **vec, _bf16_keys=np.array(bf))
    print("fixtures written")


if __name__ == "__main__":
    main()
