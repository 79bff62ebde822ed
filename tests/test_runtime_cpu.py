"""Host-side runtime logic without a GPU (reference tests/unit/test_device_kernel_cc.py,
test_device_kernel_cache.py, test_collectives.py)."""

import os
import socket
from unittest import mock

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200 import workloads as W
from nkipy_b200.runtime import compile as C
from nkipy_b200.runtime import device_kernel as DK

BF16 = np.dtype(ml_dtypes.bfloat16)


def _graph(shape=(4, 8)):
    _, g = C.specialize(W.softmax_kernel, (np.zeros(shape, np.float32),), {})
    return g


def test_graph_hash_deterministic_and_shape_sensitive():
    assert C.graph_hash(_graph()) == C.graph_hash(_graph())
    assert C.graph_hash(_graph()) != C.graph_hash(_graph((4, 16)))
    assert C.graph_hash(_graph(), world=1) != C.graph_hash(_graph(), world=2)


def test_plan_cache_reuses_files(tmp_path):
    p1, k1 = DK.DeviceKernel._trace_and_compile(W.softmax_kernel, "sm", (np.zeros((4, 8), np.float32),), {}, True, str(tmp_path), 1)
    m1 = os.path.getmtime(p1)
    p2, k2 = DK.DeviceKernel._trace_and_compile(W.softmax_kernel, "sm", (np.zeros((4, 8), np.float32),), {}, True, str(tmp_path), 1)
    assert p1 == p2 and k1 == k2 and os.path.getmtime(p2) == m1


class FakeDist:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world
        self.broadcasts, self.barriers = [], 0

    def is_available(self):
        return True

    def is_initialized(self):
        return True

    def get_world_size(self):
        return self.world

    def get_rank(self):
        return self.rank

    def broadcast_object_list(self, obj, src=0):
        self.broadcasts.append(list(obj))
        if self.rank != 0:
            obj[0], obj[1] = "/shared/plan.nkbplan", "sm_abc"

    def barrier(self):
        self.barriers += 1


@pytest.mark.parametrize("rank", [0, 1])
def test_spmd_rank0_plans_and_broadcasts(rank, tmp_path):
    fd = FakeDist(rank, 2)
    loaded = {}

    def fake_load(cls, path, name=None, **kw):
        loaded.update(path=str(path), kw=kw)
        return "kernel"

    DK._LOADED_KERNELS.clear()
    with mock.patch.object(DK, "_dist", return_value=fd), mock.patch.object(
        DK.DeviceKernel, "load_from_neff", classmethod(fake_load)
    ), mock.patch.object(DK.DeviceKernel, "_trace_and_compile", return_value=("/r0/plan.nkbplan", "sm_r0")) as tc:
        k = DK.DeviceKernel.compile_and_load(W.softmax_kernel, np.zeros((4, 8), np.float32), build_dir=str(tmp_path))
    assert k == "kernel"
    assert fd.barriers == 1 and len(fd.broadcasts) == 1
    assert tc.call_count == (1 if rank == 0 else 0)
    assert loaded["kw"] == {"cc_enabled": True, "rank_id": rank, "world_size": 2}
    assert loaded["path"] == ("/r0/plan.nkbplan" if rank == 0 else "/shared/plan.nkbplan")


def test_mpmd_builds_per_rank_directories(tmp_path):
    fd = FakeDist(1, 2)
    seen = {}

    def fake_tc(kernel, name, args, kwargs, use_cached, build_dir, world, extra=None):
        seen["dir"] = build_dir
        return ("/x/plan.nkbplan", "k")

    DK._LOADED_KERNELS.clear()
    with mock.patch.object(DK, "_dist", return_value=fd), mock.patch.object(
        DK.DeviceKernel, "_trace_and_compile", side_effect=fake_tc
    ), mock.patch.object(DK.DeviceKernel, "load_from_neff", classmethod(lambda cls, p, name=None, **kw: "k")):
        DK.DeviceKernel.compile_and_load(W.softmax_kernel, np.zeros((2, 2), np.float32), is_spmd=False,
                                         build_dir=str(tmp_path))
    assert seen["dir"].endswith("rank_1") and fd.broadcasts == [] and fd.barriers == 0


def test_cc_without_rank_world_raises():
    with mock.patch.object(DK, "_dist", return_value=None), mock.patch.object(DK, "_is_distributed", return_value=False):
        with pytest.raises(ValueError):
            DK.DeviceKernel.compile_and_load(W.softmax_kernel, np.zeros((2, 2), np.float32), cc_enabled=True)


def test_collective_plan_world_mismatch_rejected():
    s = W.LayerShape(batch=1, seq=16, hidden=128, n_heads=4, n_kv_heads=2, head_dim=32, ffn=256)
    shard = W.shard_layer_weights(W.layer_weights(s), s, 0, 2)
    args, kw = W.layer_args(np.zeros((1, 16, 128), BF16), shard, s, 2)
    _, g = C.specialize(W.llama_decoder_layer_kernel, args, kw)
    from nkipy_b200.planner import lower

    with pytest.raises(ValueError):
        lower(g, world=1)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist

    from nkipy_b200 import workloads as W
    from nkipy_b200.core.ops import collectives as cc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        s = W.LayerShape(batch=1, seq=32, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512)
        full = W.layer_weights(s, seed=3)
        x = np.random.default_rng(4).standard_normal((1, 32, 256), dtype=np.float32).astype(W.bfloat16)
        shard = W.shard_layer_weights(full, s, rank, world)
        args, kw = W.layer_args(x, shard, s, world)

        def gloo_all_reduce(data, replica_groups, reduce_op=np.add, **_):
            t = torch.from_numpy(np.asarray(data, np.float32).copy())
            dist.all_reduce(t)
            return t.numpy().astype(data.dtype)

        with mock.patch.object(cc, "all_reduce", gloo_all_reduce):
            y = W.llama_decoder_layer_kernel(*args, **kw)
        ref_args, ref_kw = W.layer_args(x, W.shard_layer_weights(full, s, 0, 1), s, 1)
        y1 = W.llama_decoder_layer_kernel(*ref_args, **ref_kw)
        err = float(np.max(np.abs(np.asarray(y, np.float32) - np.asarray(y1, np.float32))) / np.max(np.abs(np.asarray(y1, np.float32))))
        q.put((rank, err))
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_decomposition_gloo_world2():
    """Column/row sharding + one all-reduce per block reproduces TP=1 (CPU, gloo)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_tp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    assert res[0] < 2e-2 and res[1] < 2e-2, res


def _decode_worker(rank, world, port, q):
    """Vocabulary-parallel greedy sampling and a head-parallel KV-cache decode,
    the collectives done by gloo, against the single-rank direct calls."""
    import torch
    import torch.distributed as dist

    from nkipy_b200 import workloads as W
    from nkipy_b200.core.ops import collectives as cc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        def gloo_all_gather(data, all_gather_dim, replica_groups, **_):
            a = np.asarray(data)
            wide = np.float64 if a.dtype.kind == "f" or a.dtype == W.bfloat16 else np.int64
            t = torch.from_numpy(a.astype(wide))
            parts = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(parts, t)
            return np.concatenate([p.numpy() for p in parts], axis=all_gather_dim).astype(a.dtype)

        def gloo_all_reduce(data, replica_groups, reduce_op=np.add, **_):
            t = torch.from_numpy(np.asarray(data, np.float32).copy())
            dist.all_reduce(t)
            return t.numpy().astype(data.dtype)

        rng = np.random.default_rng(21)
        B, S, H, V = 3, 4, 128, 600
        h = rng.standard_normal((B, S, H), dtype=np.float32).astype(W.bfloat16)
        nw = np.ones(H, W.bfloat16)
        lm = (rng.standard_normal((H, V), dtype=np.float32) * 0.05).astype(W.bfloat16)
        shard = lm[:, rank * (V // world):(rank + 1) * (V // world)]
        with mock.patch.object(cc, "all_gather", gloo_all_gather):
            ids = W.greedy_sampling_kernel(h, nw, shard, max_batch_size=B, tp_world=world)
        full = W.greedy_sampling_kernel(h, nw, lm, max_batch_size=B, tp_world=1)
        same_ids = bool(np.array_equal(np.asarray(ids).reshape(-1), np.asarray(full).reshape(-1)))

        B, L, nq, nkv, hd, D, S = 1, 16, 4, 2, 32, 128, 4
        x = rng.standard_normal((B, S, D), dtype=np.float32).astype(W.bfloat16)
        wqkv = (rng.standard_normal((D, (nq + 2 * nkv) * hd), dtype=np.float32) * 0.05).astype(W.bfloat16)
        wo = (rng.standard_normal((nq * hd, D), dtype=np.float32) * 0.05).astype(W.bfloat16)
        qn = np.ones(hd, W.bfloat16)
        t1 = rng.standard_normal((B, 1, D), dtype=np.float32).astype(W.bfloat16)
        kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
        ck, cv = np.zeros((B, L, nkv, hd), W.bfloat16), np.zeros((B, L, nkv, hd), W.bfloat16)
        W.cached_attention_kernel(x, wqkv, qn, qn, ck, cv, None, wo, **kw)
        want = np.asarray(W.cached_attention_kernel(t1, wqkv, qn, qn, ck, cv, np.array([S], np.int32), wo, **kw),
                          np.float32)
        lq, lkv = nq // world, nkv // world
        cols = np.r_[rank * lq * hd:(rank + 1) * lq * hd,
                     nq * hd + rank * lkv * hd:nq * hd + (rank + 1) * lkv * hd,
                     (nq + nkv) * hd + rank * lkv * hd:(nq + nkv) * hd + (rank + 1) * lkv * hd]
        wr, wor = wqkv[:, cols], wo[rank * lq * hd:(rank + 1) * lq * hd]
        ckr, cvr = np.zeros((B, L, lkv, hd), W.bfloat16), np.zeros((B, L, lkv, hd), W.bfloat16)
        with mock.patch.object(cc, "all_reduce", gloo_all_reduce):
            W.cached_attention_kernel(x, wr, qn, qn, ckr, cvr, None, wor, tp_world=world, **kw)
            got = np.asarray(W.cached_attention_kernel(t1, wr, qn, qn, ckr, cvr, np.array([S], np.int32), wor,
                                                       tp_world=world, **kw), np.float32)
        err = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
        cache_ok = bool(np.array_equal(ckr.view(np.uint16), ck[:, :, rank * lkv:(rank + 1) * lkv].view(np.uint16)))
        q.put((rank, (same_ids, err, cache_ok)))
    finally:
        dist.destroy_process_group()


def test_vocab_and_head_parallel_decode_gloo_world2():
    """Greedy sampling over a vocabulary split in two (top-1 per rank, all-gather,
    top-1 over ranks) picks the same tokens as one rank; the KV-cache decode
    split by heads (+ all-reduce) matches one rank (CPU, gloo)."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_decode_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    res = dict(q.get(timeout=5) for _ in range(2))
    assert all(p.exitcode == 0 for p in procs)
    for rank in (0, 1):
        same_ids, err, cache_ok = res[rank]
        assert same_ids and cache_ok and err < 2e-2, res
