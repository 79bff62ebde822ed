"""The tracer reproduces the reference tracer's graphs, promotion and aliasing.

Fixtures were produced by the reference's own tracer (tests/golden/make_golden.py).
"""

import json
import os
import sys

import ml_dtypes
import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import golden_kernels as G  # noqa: E402

import nkipy_b200.core.ops as _ops  # noqa: E402

G.OPS = _ops

from nkipy_b200.core import graph as GR  # noqa: E402
from nkipy_b200.core.trace import NKIPyKernel  # noqa: E402

with open(os.path.join(HERE, "golden", "oplists.json")) as f:
    OPLISTS = json.load(f)
with open(os.path.join(HERE, "golden", "promotion.json")) as f:
    PROMOTION = json.load(f)


@pytest.mark.parametrize("case", G.CASES, ids=[c[0] for c in G.CASES])
def test_graph_matches_reference(case):
    name, fn, make, kw = case
    g = NKIPyKernel.trace(fn).specialize(*make(), **kw)
    got = json.loads(json.dumps(G.describe(g), sort_keys=True))
    want = OPLISTS[name]
    assert got["params"] == want["params"]
    assert [o["op"] for o in got["ops"]] == [o["op"] for o in want["ops"]]
    assert got["ops"] == want["ops"]
    assert got["results"] == want["results"]
    assert got["aliases"] == want["aliases"]


def _keys():
    return {
        "bool": np.bool_,
        "weak_int": GR._WeakInt,
        "weak_float": GR._WeakFloat,
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


def test_promotion_table_matches_reference():
    keys = _keys()
    mismatches = []
    for pair, want in PROMOTION.items():
        a, b = pair.split(",")
        try:
            r = GR._promote_keys(keys[a], keys[b])
            got = None if r is None else np.dtype(r).name
        except TypeError:
            got = "TypeError"
        if got != want:
            mismatches.append((pair, got, want))
    assert not mismatches, mismatches[:10]


def test_output_naming_and_alias():
    def k(cache, upd):
        cache[:, 1:3] = upd
        return upd * 2.0

    g = NKIPyKernel.trace(k).specialize(np.zeros((2, 5), np.float32), np.ones((2, 2), np.float32))
    assert [p.name for p in g.parameters] == ["cache.must_alias_input", "upd"]
    assert [r.name for r in g.results] == ["output0", "cache"]
    assert g.auto_aliased_indices == {1}


def test_passthrough_output_gets_copy():
    g = NKIPyKernel.trace(lambda x: x).specialize(np.zeros(3, np.float32))
    assert g.op_names() == ["copy"]


def test_int64_input_downcast_warns():
    with pytest.warns(UserWarning):
        g = NKIPyKernel.trace(lambda x: x + 1).specialize(np.zeros(3, np.int64))
    assert np.dtype(g.parameters[0].dtype) == np.int32


def test_einsum_not_registered():
    with pytest.raises(NotImplementedError):
        NKIPyKernel.trace(lambda a, b: np.einsum("ij,jk->ik", a, b)).specialize(
            np.zeros((2, 2), np.float32), np.zeros((2, 2), np.float32)
        )


def test_boolean_index_rejected():
    with pytest.raises(NotImplementedError):
        NKIPyKernel.trace(lambda a, m: a[m]).specialize(np.zeros(4, np.float32), np.zeros(4, bool))


def test_direct_call_is_numpy():
    k = NKIPyKernel.trace(G.softmax_kernel)
    x = np.random.default_rng(0).standard_normal((3, 5), dtype=np.float32)
    np.testing.assert_array_equal(k(x), G.softmax_kernel(x))
