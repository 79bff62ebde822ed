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
