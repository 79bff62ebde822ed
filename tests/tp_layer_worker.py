"""One rank of the tensor-parallel decoder-layer parity check (launched by torchrun).

Each rank plans its shard of the layer with the collective world size, runs it
through DeviceKernel (NCCL all-reduce inside the plan) and rank 0 compares the
result with the TP=1 oracle.  Exit status 0 = parity within 2e-2.
"""

import datetime
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from nkipy_b200 import workloads as W  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor
    from oracle import numpy_ref as O

    s = W.LayerShape(batch=2, seq=128, hidden=512, n_heads=8, n_kv_heads=4, head_dim=64, ffn=1024)
    full = W.layer_weights(s, seed=5)
    x = np.random.default_rng(6).standard_normal((s.batch, s.seq, s.hidden), dtype=np.float32).astype(W.bfloat16)
    shard = W.shard_layer_weights(full, s, rank, world)
    args, kw = W.layer_args(x, shard, s, world)
    k = DeviceKernel.compile_and_load(W.llama_decoder_layer_kernel, *args, name="tp_layer", is_spmd=False,
                                      cc_enabled=True, rank_id=rank, world_size=world, **kw)
    names = [t["name"] for t in k.model_ref.io["inputs"]]
    ins = {n: DeviceTensor.from_numpy(a, name=n) for n, a in zip(names, args)}
    outs = k(inputs=ins)
    y = next(iter(outs.values())).numpy().astype(np.float32)
    ok = True
    if rank == 0:
        want = O.llama_layer(x, full, s.n_heads, s.n_kv_heads, s.head_dim, s.eps, s.theta).astype(np.float32)
        err = float(np.max(np.abs(y - want)) / np.max(np.abs(want)))
        print(f"tp{world} layer rel err {err:.3e}", flush=True)
        ok = err < 2e-2
    flag = torch.tensor([1 if ok else 0])
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    dist.destroy_process_group()
    sys.exit(0 if flag.item() == 1 else 1)


if __name__ == "__main__":
    main()
