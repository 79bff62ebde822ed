"""One rank of the collective parity checks (launched by torchrun on 2+ GPUs).

* all-gather, reduce-scatter and all-to-all planned for the world size, on
  leading and inner axes, with data that differs per rank; every rank checks
  its result exactly against NumPy over all ranks' data;
* greedy sampling with the vocabulary split across the ranks
  (``examples/models/qwen3/kernels/sampling.py:113-147``: top-1 per rank,
  all-gather, top-1 over the ranks): the token chosen must hold the largest
  logit of the whole vocabulary (within the bf16 rounding of the logits);
* the Qwen3 attention block with its KV cache split by heads, a prefill and
  two decode steps with the caches resident and bound in place; rank 0
  compares every output with the single-rank NumPy direct call.

Exit status 0 = all checks pass on every rank.
"""

import datetime
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from nkipy_b200 import workloads as W  # noqa: E402
from nkipy_b200.core.ops import collectives as cc  # noqa: E402


def rank_data(r, shape=(8, 12)):
    return (np.arange(int(np.prod(shape)), dtype=np.float32).reshape(shape) + 1000.0 * r).astype(np.float32)


def check_collectives(rank, world, DeviceKernel, DeviceTensor):
    ok = True
    g = [list(range(world))]
    data = [rank_data(r) for r in range(world)]
    cases = {
        "ag0": (lambda x: cc.all_gather(x, all_gather_dim=0, replica_groups=g), np.concatenate(data, axis=0)),
        "ag1": (lambda x: cc.all_gather(x, all_gather_dim=1, replica_groups=g), np.concatenate(data, axis=1)),
        "rs0": (lambda x: cc.reduce_scatter(x, reduce_scatter_dim=0, replica_groups=g),
                np.split(sum(data), world, axis=0)[rank]),
        "rs1": (lambda x: cc.reduce_scatter(x, reduce_scatter_dim=1, replica_groups=g),
                np.split(sum(data), world, axis=1)[rank]),
        "a2a0": (lambda x: cc.all_to_all(x, split_dimension=0, concat_dimension=0, replica_groups=g),
                 np.concatenate([np.split(d, world, axis=0)[rank] for d in data], axis=0)),
        "a2a1": (lambda x: cc.all_to_all(x, split_dimension=1, concat_dimension=1, replica_groups=g),
                 np.concatenate([np.split(d, world, axis=1)[rank] for d in data], axis=1)),
    }
    for name, (fn, want) in cases.items():
        x = data[rank]
        k = DeviceKernel.compile_and_load(fn, x, name=f"cc_{name}", is_spmd=False, cc_enabled=True, rank_id=rank,
                                          world_size=world)
        outs = k(inputs={"x": DeviceTensor.from_numpy(x, name="x")})
        got = next(iter(outs.values())).numpy()
        good = got.shape == want.shape and bool(np.array_equal(got, want))
        print(f"rank {rank}: {name} exact={good}", flush=True)
        ok = ok and good
    return ok


def check_sampling(rank, world, DeviceKernel, DeviceTensor):
    B, S, H, V = 4, 8, 512, 4000
    rng = np.random.default_rng(11)
    h = rng.standard_normal((B, S, H), dtype=np.float32).astype(W.bfloat16)
    nw = rng.uniform(0.5, 1.5, H).astype(W.bfloat16)
    lm = (rng.standard_normal((H, V), dtype=np.float32) * 0.05).astype(W.bfloat16)
    shard = np.ascontiguousarray(lm[:, rank * (V // world):(rank + 1) * (V // world)])
    kw = dict(max_batch_size=B, tp_world=world)
    k = DeviceKernel.compile_and_load(W.greedy_sampling_kernel, h, nw, shard, name="tp_sampling", is_spmd=False,
                                      cc_enabled=True, rank_id=rank, world_size=world, **kw)
    names = [t["name"] for t in k.model_ref.io["inputs"]]
    outs = k(inputs={n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(names, (h, nw, shard))})
    ids = next(iter(outs.values())).numpy().reshape(-1).astype(np.int64)
    hn = W.qk_rmsnorm(h, nw, 1e-6)
    logits = hn[:, -1, :].astype(np.float32) @ lm.astype(np.float32)
    best = logits.max(axis=1)
    tol = 2.0 ** -7 * np.abs(best) + 1e-6
    picked = logits[np.arange(B), np.clip(ids, 0, V - 1)]
    good = bool(np.all((ids >= 0) & (ids < V)) and np.all(picked >= best - tol))
    print(f"rank {rank}: tp{world} greedy sampling ids={ids.tolist()} argmax={logits.argmax(1).tolist()} ok={good}",
          flush=True)
    return good


def check_cached_attention(rank, world, DeviceKernel, DeviceTensor):
    B, L, nq, nkv, hd, D, S = 2, 64, 8, 2 * world, 64, 512, 16
    rng = np.random.default_rng(12)
    x = rng.standard_normal((B, S, D), dtype=np.float32).astype(W.bfloat16)
    wqkv = (rng.standard_normal((D, (nq + 2 * nkv) * hd), dtype=np.float32) * 0.02).astype(W.bfloat16)
    wo = (rng.standard_normal((nq * hd, D), dtype=np.float32) * 0.02).astype(W.bfloat16)
    qn = rng.uniform(0.5, 1.5, hd).astype(W.bfloat16)
    kn = rng.uniform(0.5, 1.5, hd).astype(W.bfloat16)
    toks = [rng.standard_normal((B, 1, D), dtype=np.float32).astype(W.bfloat16) for _ in range(2)]
    kw = dict(n_heads=nq, head_dim=hd, n_kv_heads=nkv)
    # single-rank reference (NumPy direct call)
    ck, cv = np.zeros((B, L, nkv, hd), W.bfloat16), np.zeros((B, L, nkv, hd), W.bfloat16)
    want = [W.cached_attention_kernel(x, wqkv, qn, kn, ck, cv, None, wo, **kw)]
    for i, t in enumerate(toks):
        want.append(W.cached_attention_kernel(t, wqkv, qn, kn, ck, cv, np.array([S + i], np.int32), wo, **kw))
    # this rank's heads: q heads, kv heads, o rows (examples/models/qwen3/tensor_preparation.py:15-31)
    lq, lkv = nq // world, nkv // world
    qc = slice(rank * lq * hd, (rank + 1) * lq * hd)
    kc = slice(nq * hd + rank * lkv * hd, nq * hd + (rank + 1) * lkv * hd)
    vc = slice((nq + nkv) * hd + rank * lkv * hd, (nq + nkv) * hd + (rank + 1) * lkv * hd)
    wqkv_r = np.ascontiguousarray(np.concatenate([wqkv[:, qc], wqkv[:, kc], wqkv[:, vc]], axis=1))
    wo_r = np.ascontiguousarray(wo[qc, :])
    z = np.zeros((B, L, lkv, hd), W.bfloat16)
    kwr = dict(kw, tp_world=world)
    common = dict(is_spmd=False, cc_enabled=True, rank_id=rank, world_size=world)
    pre = DeviceKernel.compile_and_load(W.cached_attention_kernel, x, wqkv_r, qn, kn, z, z, None, wo_r,
                                        name="tp_cache_prefill", **common, **kwr)
    dec = DeviceKernel.compile_and_load(W.cached_attention_kernel, toks[0], wqkv_r, qn, kn, z, z,
                                        np.array([S], np.int32), wo_r, name="tp_cache_decode", **common, **kwr)
    dk, dv = DeviceTensor.from_numpy(z), DeviceTensor.from_numpy(z)
    w = {n: DeviceTensor.from_numpy(a) for n, a in
         (("qkv_weight", wqkv_r), ("q_norm_weight", qn), ("k_norm_weight", kn), ("o_weight", wo_r))}
    cache = {"cache_k.must_alias_input": dk, "cache_v.must_alias_input": dv}
    y = DeviceTensor.empty((B, S, D), W.bfloat16)
    pre(inputs=dict(w, x=DeviceTensor.from_numpy(x), **cache), outputs={"output0": y, "cache_k": dk, "cache_v": dv})
    got = [y.numpy()]
    y1 = DeviceTensor.empty((B, 1, D), W.bfloat16)
    for i, t in enumerate(toks):
        pos = DeviceTensor.from_numpy(np.array([S + i], np.int32))
        dec(inputs=dict(w, x=DeviceTensor.from_numpy(t), start_pos=pos, **cache),
            outputs={"output0": y1, "cache_k": dk, "cache_v": dv})
        got.append(y1.numpy())
    errs = []
    for g_, e in zip(got, want):
        g_, e = g_.astype(np.float32), np.asarray(e, np.float32)
        errs.append(float(np.max(np.abs(g_ - e)) / np.max(np.abs(e))))
    kc_want = ck[:, :, rank * lkv:(rank + 1) * lkv].astype(np.float32)
    errs.append(float(np.max(np.abs(dk.numpy().astype(np.float32) - kc_want)) / np.max(np.abs(kc_want))))
    good = all(e < 2e-2 for e in errs)
    print(f"rank {rank}: tp{world} cached attention rel errs {['%.2e' % e for e in errs]} ok={good}", flush=True)
    return good


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("cpu:gloo,cuda:nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    ok = check_collectives(rank, world, DeviceKernel, DeviceTensor)
    ok = check_sampling(rank, world, DeviceKernel, DeviceTensor) and ok
    ok = check_cached_attention(rank, world, DeviceKernel, DeviceTensor) and ok
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
