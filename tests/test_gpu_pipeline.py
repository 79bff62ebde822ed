"""Pipelined execution (``SpikeModel.run_steps``): every step uploads its inputs
from page-locked host memory, executes and reads its outputs back, with the
copies of one step overlapping the compute of the next; results must equal
the synchronous execute's, step by step, including a mutated input bound in
place as its own output."""

import numpy as np
import pytest

from nkipy_b200 import workloads as W
from oracle import numpy_ref as O
from tests.utils import FP32_RTOL, assert_close

pytestmark = pytest.mark.gpu


def _pinned(shape, dtype):
    import torch

    n = int(np.prod(shape)) * np.dtype(dtype).itemsize
    return torch.empty(n, dtype=torch.uint8, pin_memory=True).numpy().view(dtype).reshape(shape)


@pytest.mark.parametrize("steps", [1, 2, 5])
def test_run_steps_matches_each_step(steps):
    from nkipy_b200.runtime import DeviceKernel

    rng = np.random.default_rng(50)
    feeds = []
    for _ in range(3):
        a = _pinned((256, 1024), np.float32)
        a[:] = rng.standard_normal((256, 1024), dtype=np.float32)
        feeds.append(a)
    k = DeviceKernel.compile_and_load(W.softmax_kernel, feeds[0], name="pipe_softmax", is_spmd=False)
    name_in = k.model_ref.io["inputs"][0]["name"]
    name_out = k.model_ref.io["outputs"][0]["name"]
    out = _pinned((256, 1024), np.float32)
    k.run_steps({}, {name_in: feeds}, {name_out: out}, steps)
    assert_close(out, O.softmax(feeds[(steps - 1) % 3]), FP32_RTOL, atol=1e-7)


def test_run_steps_with_an_input_updated_in_place():
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    def kern(a, idx, v):
        a[:, idx] = v
        return a.sum(axis=1)

    rng = np.random.default_rng(51)
    a = rng.standard_normal((64, 40), dtype=np.float32)
    idx = np.array([7], np.int32)
    vs = []
    for _ in range(4):
        v = _pinned((64, 1), np.float32)
        v[:] = rng.standard_normal((64, 1), dtype=np.float32)
        vs.append(v)
    k = DeviceKernel.compile_and_load(kern, a.copy(), idx, vs[0], name="pipe_inplace", is_spmd=False)
    names = [t["name"] for t in k.model_ref.io["inputs"]]
    a_name = next(n for n in names if n.endswith(".must_alias_input"))
    idx_name = next(n for n in names if n.startswith("idx"))
    v_name = next(n for n in names if n.startswith("v"))
    outs = [t["name"] for t in k.model_ref.io["outputs"]]
    a_dev = DeviceTensor.from_numpy(a.copy(), name=a_name)
    sums = _pinned((64,), np.float32)
    alias_out = next(o for o in outs if f"{o}.must_alias_input" == a_name)
    sum_out = next(o for o in outs if o != alias_out)
    k.run_steps({a_name: a_dev, idx_name: DeviceTensor.from_numpy(idx, name=idx_name)}, {v_name: vs},
                {sum_out: sums}, 4, bind={alias_out: a_dev})
    want = a.copy()
    want[:, 7:8] = vs[3]
    np.testing.assert_array_equal(a_dev.numpy(), want)
    assert_close(sums, want.sum(axis=1), FP32_RTOL, atol=FP32_RTOL * np.abs(want).sum(axis=1))


def test_time_execute_steps_times_each_launch_inside_one_replay():
    """The bench's timed steps replay a graph with an event between every two
    launches: the per-launch times add up to the execute's time, and the result
    is the plan's."""
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor
    from nkipy_b200.spike import get_spike_singleton

    rng = np.random.default_rng(52)
    x = rng.standard_normal((256, 1024), dtype=np.float32)
    r = rng.standard_normal((256, 1024), dtype=np.float32)
    w = rng.uniform(0.5, 1.5, 1024).astype(np.float32)

    def kern(x, r, w):  # two launches: a residual + RMSNorm, then a softmax
        return W.softmax_kernel(W.residual_rmsnorm_kernel(x, r, w))

    k = DeviceKernel.compile_and_load(kern, x, r, w, name="timing_two_launches", is_spmd=False)
    model = k.model_ref
    names = [t["name"] for t in model.io["inputs"]]
    ins = {n: DeviceTensor.from_numpy(a, name=n).tensor_ref for n, a in zip(names, (x, r, w))}
    outs = {t.name: t.tensor_ref for t in k.allocate_output_tensors()}
    spike = get_spike_singleton()
    for _ in range(2):
        total, per = spike.time_execute_steps(model, ins, outs)
    assert len(per) == model.num_launches >= 2
    assert all(p > 0 for p in per) and total > 0
    assert abs(sum(per) - total) <= 0.05 * total + 1e-3
    got = np.frombuffer(spike.tensor_read(next(iter(outs.values()))), np.float32)[: x.size].reshape(x.shape)
    assert_close(got, O.softmax(O.residual_rmsnorm(x, r, w)), 1e-5, atol=1e-6)
