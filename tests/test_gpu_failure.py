"""Failure paths of the runtime on one GPU, none of which faults or hangs it.

* A bounded wait that expires (a counter that nothing advances, with a 2 ms
  budget) is reported by nkb_device_error, the flag clears on reading, and
  the context stays usable (the reference surfaces NRT failures as
  NrtError(status), spike/src/include/error.h:12-43).
* Use after free, out-of-range slices and copies, and plans run with the
  wrong number of tensors return status codes with messages, as Spike's
  bounds-checked tensor calls raise (spike/src/tensor.cpp:65-105).
"""

import ctypes

import numpy as np
import pytest

from nkipy_b200 import workloads as W
from nkipy_b200.spike import _nkb, get_spike_singleton
from oracle import numpy_ref as O
from tests.utils import FP32_RTOL, assert_close, on_device

pytestmark = pytest.mark.gpu

INVALID, STATE, PLAN = 1, 6, 3


def _flag():
    f = ctypes.c_int(-1)
    _nkb.call("nkb_device_error", ctypes.byref(f))
    return f.value


def test_expired_wait_is_reported_and_context_survives():
    spike = get_spike_singleton()
    lib = _nkb.lib()
    counter = spike.allocate_tensor(4)
    spike.tensor_write_from_pybuffer(counter, np.zeros(1, np.uint32))
    old = ctypes.c_uint64()
    _nkb.call("nkb_get_wait_limit_us", ctypes.byref(old))
    try:
        _nkb.call("nkb_set_wait_limit_us", 2000)
        assert _flag() == 0
        _nkb.check(lib.nkb_wait_probe(ctypes.c_void_p(counter.va), 1, None))
        _nkb.call("nkb_synchronize")
        assert _flag() == 1  # the wait ran out and said so
        assert _flag() == 0  # reading cleared it
        # the counter reaches the target: the same wait succeeds
        spike.tensor_write_from_pybuffer(counter, np.ones(1, np.uint32))
        _nkb.check(lib.nkb_wait_probe(ctypes.c_void_p(counter.va), 1, None))
        _nkb.call("nkb_synchronize")
        assert _flag() == 0
    finally:
        _nkb.call("nkb_set_wait_limit_us", old.value)
    # the context is still usable
    x = np.random.default_rng(40).standard_normal((64, 1024), dtype=np.float32)
    assert_close(on_device(W.softmax_kernel, x), O.softmax(x), FP32_RTOL)


def test_wait_limit_rejects_zero():
    get_spike_singleton()
    assert _nkb.lib().nkb_set_wait_limit_us(0) == INVALID


def test_use_after_free_and_double_free():
    get_spike_singleton()
    lib = _nkb.lib()
    h = ctypes.c_void_p()
    _nkb.call("nkb_alloc", 256, get_spike_singleton().device, ctypes.byref(h))
    s = ctypes.c_void_p()
    _nkb.call("nkb_slice", h, 0, 64, ctypes.byref(s))
    _nkb.call("nkb_free", s)
    assert lib.nkb_free(s) == STATE  # the slice is gone
    _nkb.call("nkb_free", h)
    buf = (ctypes.c_uint8 * 16)()
    assert lib.nkb_h2d(h, buf, 16, 0) == STATE
    assert b"freed" in lib.nkb_last_error()
    assert lib.nkb_d2h(h, buf, 16, 0) == STATE
    assert lib.nkb_free(h) == STATE


def test_out_of_range_slices_and_copies():
    spike = get_spike_singleton()
    lib = _nkb.lib()
    t = spike.allocate_tensor(1024)
    buf = (ctypes.c_uint8 * 2048)()
    s = ctypes.c_void_p()
    assert lib.nkb_slice(t.handle, 1000, 100, ctypes.byref(s)) == INVALID
    assert b"exceeds" in lib.nkb_last_error()
    assert lib.nkb_slice(t.handle, 2000, 0, ctypes.byref(s)) == INVALID
    assert lib.nkb_h2d(t.handle, buf, 1025, 0) == INVALID
    assert lib.nkb_h2d(t.handle, buf, 8, 1020) == INVALID
    assert lib.nkb_d2h(t.handle, buf, 2048, 0) == INVALID
    assert lib.nkb_memset(t.handle, 0, 16, 1016) == INVALID
    # a slice is bounded by its own extent, not its parent's
    _nkb.call("nkb_slice", t.handle, 512, 256, ctypes.byref(s))
    assert lib.nkb_h2d(s, buf, 257, 0) == INVALID
    _nkb.call("nkb_h2d", s, buf, 256, 0)
    _nkb.call("nkb_free", s)
    with pytest.raises(_nkb.NkbError):
        spike.tensor_write(t, b"x" * 2000)


def test_plan_run_with_wrong_tensors():
    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    x = np.random.default_rng(41).standard_normal((8, 256), dtype=np.float32)
    k = DeviceKernel.compile_and_load(W.softmax_kernel, x, name="failure_softmax", is_spmd=False)
    model = k.model_ref
    lib = _nkb.lib()
    xin = DeviceTensor.from_numpy(x, name="x").tensor_ref
    small = get_spike_singleton().allocate_tensor(16)
    out = get_spike_singleton().allocate_tensor(x.nbytes)
    I1 = (ctypes.c_void_p * 1)(xin.handle.value)
    O1 = (ctypes.c_void_p * 1)(out.handle.value)
    O2 = (ctypes.c_void_p * 2)(out.handle.value, out.handle.value)
    assert lib.nkb_execute(model.handle, I1, 1, O2, 2, None, 0) == INVALID  # output count mismatch
    assert lib.nkb_execute(model.handle, I1, 0, O1, 1, None, 0) == INVALID  # input count mismatch
    S1 = (ctypes.c_void_p * 1)(small.handle.value)
    assert lib.nkb_execute(model.handle, I1, 1, S1, 1, None, 0) != 0  # output buffer too small
    assert lib.nkb_last_error()
    # the right tensors still run
    _nkb.call("nkb_execute", model.handle, I1, 1, O1, 1, None, 0)
    _nkb.call("nkb_synchronize")


@pytest.mark.parametrize(
    "text,word",
    [
        ("NKBPLAN 1\nname t\ninputs 0\noutputs 0\nconsts 0\nscratch 0\nbuffers 0\nsteps 1\nstep no_such_kernel 0 0 0\nend\n",
         b"no_such_kernel"),
        ("NKBPLAN 1\nname t\ninputs 1\ninput 0 64\noutputs 1\noutput 0 64\nconsts 0\nscratch 0\nbuffers 2\n"
         "buffer 0 in 0\nbuffer 1 out 0\nsteps 1\nstep copy_bytes 2 0 0 1 0 2 64 64 0\nend\n", b"copy_bytes"),
        ("NOT A PLAN\n", b""),
    ],
)
def test_malformed_plans_rejected_at_load(text, word):
    get_spike_singleton()
    lib = _nkb.lib()
    h = ctypes.c_void_p()
    raw = text.encode()
    st = lib.nkb_plan_load(raw, len(raw), get_spike_singleton().device, ctypes.byref(h))
    assert st == PLAN, (st, lib.nkb_last_error())
    assert word in lib.nkb_last_error()


def test_save_trace_writes_a_launch_timeline(tmp_path):
    """save_trace=True (the reference's per-execute profile) writes a Chrome
    trace of the execute's launches, one event per kernel, next to the plan
    or at ntff_name."""
    import json

    from nkipy_b200.runtime import DeviceKernel, DeviceTensor

    x = np.random.default_rng(42).standard_normal((64, 4096), dtype=np.float32)
    k = DeviceKernel.compile_and_load(W.softmax_kernel, x, name="trace_softmax", is_spmd=False)
    name = k.model_ref.io["inputs"][0]["name"]
    path = str(tmp_path / "softmax.trace.json")
    outs = k(inputs={name: DeviceTensor.from_numpy(x, name=name)}, save_trace=True, ntff_name=path)
    with open(path) as f:
        ev = json.load(f)["traceEvents"]
    assert [e["name"] for e in ev] == ["softmax_rows"] and ev[0]["dur"] > 0
    assert_close(next(iter(outs.values())).numpy(), O.softmax(x), FP32_RTOL, atol=1e-7)
