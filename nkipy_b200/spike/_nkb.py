"""ctypes binding of libnkb.so (the C ABI declared in include/nkb.h).

Replaces the reference's nanobind module ``_spike`` (spike/src/python_bindings.cpp).
The library is loaded from the package tree (``nkipy_b200/_lib/libnkb.so``,
built by ``python -m nkipy_b200.build``); a missing library is an ImportError,
never a silent fallback.  Every call checks the returned status and raises
``NkbError(status, message)``; ctypes releases the GIL for the duration of
each foreign call, as the reference does around ``execute``
(python_bindings.cpp:121-126).
"""

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "_lib", "libnkb.so")

STATUS_NAMES = {
    0: "ok",
    1: "invalid argument",
    2: "CUDA error",
    3: "plan error",
    4: "unsupported",
    5: "NCCL error",
    6: "invalid state",
    7: "device-reported error",
}


class SpikeRuntimeError(RuntimeError):
    """Base of runtime errors (reference ``error.h:12-43``)."""


class SpikeError(SpikeRuntimeError):
    """Host-side misuse: freed handles, size mismatches (``SpikeError``)."""


class NkbError(SpikeRuntimeError):
    """A libnkb call failed; ``status`` is the C status code (``NrtError``)."""

    def __init__(self, status: int, message: str):
        self.status = status
        super().__init__(f"[{STATUS_NAMES.get(status, status)}] {message}")


NrtError = NkbError

_lib = None

c_buf = ctypes.c_void_p
c_plan = ctypes.c_void_p
c_comm = ctypes.c_void_p


def _declare(lib):
    i32, i64, sz, vp = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p
    pp = ctypes.POINTER(ctypes.c_void_p)
    sig = {
        "nkb_init": [i32],
        "nkb_shutdown": [],
        "nkb_device_count": [ctypes.POINTER(i32)],
        "nkb_version": [ctypes.POINTER(i32), ctypes.POINTER(i32)],
        "nkb_alloc": [sz, i32, pp],
        "nkb_slice": [c_buf, sz, sz, pp],
        "nkb_wrap": [vp, sz, i32, pp],
        "nkb_free": [c_buf],
        "nkb_buf_info": [c_buf, ctypes.POINTER(sz), ctypes.POINTER(i32), pp],
        "nkb_h2d": [c_buf, vp, sz, sz],
        "nkb_d2h": [c_buf, vp, sz, sz],
        "nkb_memset": [c_buf, i32, sz, sz],
        "nkb_copy": [c_buf, sz, c_buf, sz, sz],
        "nkb_plan_load": [ctypes.c_char_p, sz, i32, pp],
        "nkb_plan_free": [c_plan],
        "nkb_plan_num_io": [c_plan, ctypes.POINTER(i32), ctypes.POINTER(i32)],
        "nkb_plan_io_bytes": [c_plan, i32, i32, ctypes.POINTER(sz)],
        "nkb_plan_num_consts": [c_plan, ctypes.POINTER(i32)],
        "nkb_plan_set_const": [c_plan, i32, vp, sz],
        "nkb_plan_num_launches": [c_plan, ctypes.POINTER(i32)],
        "nkb_plan_graph_kernels": [c_plan, ctypes.POINTER(i32)],
        "nkb_time_execute_steps": [c_plan, pp, i32, pp, i32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)],
        "nkb_plan_scratch_bytes": [c_plan, ctypes.POINTER(sz)],
        "nkb_ew_compiler_stats": [ctypes.POINTER(ctypes.c_int64)] * 3,
        "nkb_ew_compile_step": [ctypes.POINTER(ctypes.c_int64), sz, ctypes.POINTER(i32)],
        "nkb_execute": [c_plan, pp, i32, pp, i32, vp, i32],
        "nkb_time_execute": [c_plan, pp, i32, pp, i32, i32, i32, i32, ctypes.POINTER(ctypes.c_float)],
        "nkb_synchronize": [],
        "nkb_time_steps": [c_plan, pp, i32, pp, i32, i32, ctypes.POINTER(ctypes.c_float)],
        "nkb_device_error": [ctypes.POINTER(i32)],
        "nkb_trace_execute": [c_plan, pp, i32, pp, i32, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(ctypes.c_float)],
        "nkb_stream_create": [pp],
        "nkb_stream_destroy": [vp],
        "nkb_stream_synchronize": [vp],
        "nkb_event_create": [pp],
        "nkb_event_destroy": [vp],
        "nkb_event_record": [vp, vp],
        "nkb_stream_wait_event": [vp, vp],
        "nkb_h2d_async": [c_buf, vp, sz, sz, vp],
        "nkb_d2h_async": [c_buf, vp, sz, sz, vp],
        "nkb_set_wait_limit_us": [ctypes.c_uint64],
        "nkb_get_wait_limit_us": [ctypes.POINTER(ctypes.c_uint64)],
        "nkb_wait_probe": [vp, ctypes.c_uint32, vp],
        "nkb_comm_unique_id": [vp],
        "nkb_comm_init": [vp, i32, i32, i32, pp],
        "nkb_comm_free": [c_comm],
        "nkb_plan_bind_comm": [c_plan, c_comm],
        "nkb_comm_all_reduce": [c_comm, c_buf, sz, i32, vp],
        "nkb_comm_bind_symm": [c_comm, vp, vp, pp, i32, sz],
        "nkb_softmax_rows": [vp, i32, vp, i32, i64, i64, vp],
        "nkb_rmsnorm_rows": [vp, vp, vp, vp, vp, i32, i32, i64, i64, ctypes.c_float, vp],
        "nkb_gemm_bf16": [vp, vp, vp, i32, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64, vp],
        "nkb_topk_rows": [vp, i32, vp, vp, i64, i64, i64, vp],
        "nkb_comm_all_gather": [c_comm, vp, vp, sz, i32, vp],
        "nkb_comm_reduce_scatter": [c_comm, vp, vp, sz, i32, vp],
        "nkb_comm_all_to_all": [c_comm, vp, vp, sz, i32, vp],
        "nkb_linear_attention_noalloc": [vp, vp, vp, vp, i64, i64, i64, i64, vp],
    }
    for name, args in sig.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = i32
    lib.nkb_last_error.argtypes = []
    lib.nkb_last_error.restype = ctypes.c_char_p
    lib.nkb_status_str.argtypes = [ctypes.c_int]
    lib.nkb_status_str.restype = ctypes.c_char_p
    lib.nkb_comm_symm_flag_bytes.argtypes = []
    lib.nkb_comm_symm_flag_bytes.restype = ctypes.c_size_t
    return sorted(sig) + ["nkb_last_error", "nkb_status_str", "nkb_comm_symm_flag_bytes"]


EXPORTED = None


def lib():
    """Load libnkb once; raise ImportError when it has not been built."""
    global _lib, EXPORTED
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libnkb.so not found at {LIB_PATH}; build it with `python -m nkipy_b200.build`")
        handle = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_GLOBAL)
        EXPORTED = _declare(handle)
        _lib = handle
    return _lib


def check(status: int):
    if status != 0:
        msg = lib().nkb_last_error()
        raise NkbError(status, msg.decode() if msg else "")


def call(name, *args):
    check(getattr(lib(), name)(*args))
