"""The allocation-free linear-attention entry point agrees with the planned path
(and with the CPU oracle).

``nkb_linear_attention_noalloc`` exists for callers that cannot allocate device
memory when they run the kernel (a host whose caching allocator owns the whole
GPU, or a latency-critical loop where cudaMalloc/cudaFree could block or
synchronise the device): the caller passes only inputs and the output, and
the kernel's workspace is a fixed device array inside libnkb.  This test calls
it through the C ABI twice in a row on the same buffers and compares each
result with the existing entry point (the planned kernel run by nkb_execute)
within the bf16 tolerance of the other GPU tests; the last result is also
compared with the oracle on one (batch, head) pair.
"""

import ctypes

import ml_dtypes
import numpy as np
import pytest

from nkipy_b200 import workloads as W
from nkipy_b200.core.trace import NKIPyKernel
from nkipy_b200.runtime import baremetal_run_traced_kernel
from nkipy_b200.spike import _nkb, get_spike_singleton
from tests.utils import BF16_RTOL, assert_close

BF16 = np.dtype(ml_dtypes.bfloat16)
pytestmark = pytest.mark.gpu


def test_noalloc_linear_attention_matches_planned_path():
    import torch

    B, H, T, D = 2, 4, 3072, 128  # 3 segments: exercises the workspace and the scan
    rng = np.random.default_rng(21)
    q, k, v = (rng.standard_normal((B, H, T, D), dtype=np.float32).astype(BF16) for _ in range(3))

    # existing entry point: the traced kernel planned and run through nkb_execute
    want = baremetal_run_traced_kernel(NKIPyKernel.trace(W.chunked_linear_attention_kernel), q, k, v)

    spike = get_spike_singleton()
    dev = [spike.allocate_tensor(a.nbytes) for a in (q, k, v)]
    for t, a in zip(dev, (q, k, v)):
        spike.tensor_write_from_pybuffer(t, a)
    out = spike.allocate_tensor(q.nbytes)
    lib = _nkb.lib()
    for _ in range(2):
        spike.tensor_write_from_pybuffer(out, np.zeros_like(q))
        st = lib.nkb_linear_attention_noalloc(
            ctypes.c_void_p(dev[0].va), ctypes.c_void_p(dev[1].va), ctypes.c_void_p(dev[2].va),
            ctypes.c_void_p(out.va), B, H, T, D, None,
        )
        _nkb.check(st)
        torch.cuda.synchronize()
        got = np.empty_like(q)
        spike.tensor_read_to_pybuffer(out, got)
        assert_close(got, want, BF16_RTOL)
        flag = ctypes.c_int()
        _nkb.call("nkb_device_error", ctypes.byref(flag))
        assert flag.value == 0  # no bounded wait of the kernel expired
    # and against the CPU oracle (the recurrent form) on one (batch, head) pair
    from oracle import numpy_ref as O

    sl = (slice(1, 2), slice(3, 4))
    assert_close(got[sl], O.linear_attention_recurrent(q[sl], k[sl], v[sl]), BF16_RTOL)


def test_noalloc_rejects_oversized_workspace():
    import torch

    lib = _nkb.lib()
    get_spike_singleton()
    # 4 heads of 262144 tokens need 256 segment states each (67.6 MB), more
    # than the fixed array; the size check happens before any memory is touched.
    fake = ctypes.c_void_p(256)
    st = lib.nkb_linear_attention_noalloc(fake, fake, fake, fake, 1, 4, 262144, 128, None)
    assert st == 1 and b"workspace" in lib.nkb_last_error()
    torch.cuda.synchronize()
