"""One rank of the tensor-parallel decoder-layer parity check (launched by torchrun).

Each rank plans its shard of the layer with the collective world size, runs it
through DeviceKernel (all-reduce inside the plan: inside NVSwitch when a
symmetric region could be bound, NCCL otherwise, or NCCL only with
NKB_SYMM=0) and rank 0 compares the result with the TP=1 oracle.  Before
that, the plan's communicator all-reduces a buffer of small integers whose sum
is exact in bf16, and a GEMM + all-reduce + residual plan on small integers
is compared exactly with NumPy.  Exit status 0 = all checks pass.
"""

import ctypes
import datetime
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from nkipy_b200 import workloads as W  # noqa: E402
from nkipy_b200.core.ops import collectives as cc  # noqa: E402


def check_all_reduce(model, rank, world):
    """The communicator bound to the plan sums exactly representable bf16 values
    (in the bound symmetric region when there is one, so inside NVSwitch)."""
    from nkipy_b200.spike import _nkb
    from nkipy_b200.spike import runtime as R

    n = 1 << 20
    i = np.arange(n)
    x = ((i % 64) + rank).astype(W.bfloat16)
    h = ctypes.c_void_p()
    if model.symmetric:
        region = R._SYMM[(world, rank)][1][-2]  # the bound symmetric tensor
        _nkb.call("nkb_wrap", ctypes.c_void_p(region.data_ptr()), n * 2, local_device(), ctypes.byref(h))
    else:
        _nkb.call("nkb_alloc", n * 2, local_device(), ctypes.byref(h))
    _nkb.call("nkb_h2d", h, x.ctypes.data_as(ctypes.c_void_p), n * 2, 0)
    _nkb.call("nkb_comm_all_reduce", model.comm, h, n, 1, None)
    _nkb.call("nkb_synchronize")
    got = np.empty_like(x)
    _nkb.call("nkb_d2h", h, got.ctypes.data_as(ctypes.c_void_p), n * 2, 0)
    _nkb.call("nkb_free", h)
    want = (world * (i % 64) + world * (world - 1) // 2).astype(np.float32)
    flag = ctypes.c_int()
    _nkb.call("nkb_device_error", ctypes.byref(flag))
    ok = bool(np.array_equal(got.astype(np.float32), want)) and flag.value == 0
    print(f"rank {rank}: all-reduce {'NVLS' if model.symmetric else 'NCCL'} exact={ok}", flush=True)
    return ok


def gemm_all_reduce_kernel(a, b, r, world=2):
    """A row-parallel GEMM, its all-reduce and the residual add after it."""
    p = a @ b
    s = cc.all_reduce(p, replica_groups=[list(range(world))], reduce_op=np.add)
    return r + s


def gemm_ar_inputs(rank, M=1000, K=384, N=520):
    """Small integers whose products, sums over the ranks and residual add are exact in bf16."""
    g = np.random.default_rng(100 + rank)
    a = g.integers(-1, 2, (M, K)) * (g.random((M, K)) < 1 / 64)
    b = g.integers(-1, 2, (K, N))
    r = np.random.default_rng(99).integers(-32, 33, (M, N))
    return [x.astype(np.float32).astype(W.bfloat16) for x in (a, b, r)]


def check_gemm_all_reduce(rank, world):
    """gemm_bf16_ar (fused in the GEMM when a symmetric region is bound) over a
    ragged shape: 8 row blocks, the last of 104 rows, and a partial last column tile."""
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    a, b, r = gemm_ar_inputs(rank)
    k = DeviceKernel.compile_and_load(gemm_all_reduce_kernel, a, b, r, world=world, name="tp_gemm_ar", is_spmd=False,
                                      cc_enabled=True, rank_id=rank, world_size=world)
    kinds = k.model_ref.io["kernels"]
    names = [t["name"] for t in k.model_ref.io["inputs"]]
    outs = k(inputs={n: DeviceTensor.from_numpy(x, name=n) for n, x in zip(names, (a, b, r))})
    got = next(iter(outs.values())).numpy().astype(np.float32)
    want = r.astype(np.float32).copy()
    for q in range(world):
        aq, bq, _ = gemm_ar_inputs(q)
        want += aq.astype(np.float32) @ bq.astype(np.float32)
    flag = ctypes.c_int()
    from nkipy_b200.spike import _nkb

    _nkb.call("nkb_device_error", ctypes.byref(flag))
    ok = kinds.get("gemm_bf16_ar") == 1 and bool(np.array_equal(got, want)) and flag.value == 0
    print(f"rank {rank}: gemm + all-reduce + residual exact={ok} ({kinds})", flush=True)
    return ok


def local_device():
    return int(os.environ.get("LOCAL_RANK", os.environ["RANK"]))


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor
    from oracle import numpy_ref as O

    kv = max(4, world)  # whole kv heads per rank
    s = W.LayerShape(batch=2, seq=128, hidden=128 * kv, n_heads=2 * kv, n_kv_heads=kv, head_dim=64, ffn=256 * kv)
    full = W.layer_weights(s, seed=5)
    x = np.random.default_rng(6).standard_normal((s.batch, s.seq, s.hidden), dtype=np.float32).astype(W.bfloat16)
    shard = W.shard_layer_weights(full, s, rank, world)
    args, kw = W.layer_args(x, shard, s, world)
    k = DeviceKernel.compile_and_load(W.llama_decoder_layer_kernel, *args, name="tp_layer", is_spmd=False,
                                      cc_enabled=True, rank_id=rank, world_size=world, **kw)
    model = k.model_ref
    ok = check_all_reduce(model, rank, world)
    ok = check_gemm_all_reduce(rank, world) and ok
    names = [t["name"] for t in model.io["inputs"]]
    ins = {n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(names, args)}
    outs = k(inputs=ins)
    y = next(iter(outs.values())).numpy().astype(np.float32)
    if rank == 0:
        want = O.llama_layer(x, full, s.n_heads, s.n_kv_heads, s.head_dim, s.eps, s.theta).astype(np.float32)
        err = float(np.max(np.abs(y - want)) / np.max(np.abs(want)))
        print(f"tp{world} layer rel err {err:.3e}", flush=True)
        ok = ok and err < 2e-2
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
