"""Multi-GPU tests (2 GPUs): the tensor-parallel decoder layer with its all-reduce inside NVSwitch (own
kernel) and through NCCL; the other collectives, vocabulary-parallel sampling and a head-parallel KV cache."""

import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch

        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("symm", ["force", "0"], ids=["nvswitch", "nccl"])
def test_tp2_layer_parity(symm):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NKB_SYMM=symm)
    cmd = [
        "timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
        os.path.join(ROOT, "tests", "tp_layer_worker.py"),
    ]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_tp2_collectives_sampling_and_kv_cache():
    """all-gather / reduce-scatter / all-to-all, vocabulary-parallel greedy
    sampling and the head-parallel KV-cache decode on 2 GPUs (NCCL)."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [
        "timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
        "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29541",
        os.path.join(ROOT, "tests", "collectives_worker.py"),
    ]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
