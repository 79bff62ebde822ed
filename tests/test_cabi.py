"""The C ABI library loads and exports every entry point of include/nkb.h.

No compute calls: this runs without a GPU.  Error paths return status codes
with messages instead of crashing.
"""

import ctypes
import os
import re

import pytest

from nkipy_b200.spike import _nkb

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "nkb.h")


def declared():
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"NKB_API\s+[^;(]*?\b(nkb_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared()
    assert "nkb_execute" in names and "nkb_plan_load" in names and len(names) >= 30


def test_library_exports_every_declared_symbol():
    lib = _nkb.lib()
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_python_binding_covers_header():
    _nkb.lib()
    assert set(declared()) <= set(_nkb.EXPORTED)


def test_status_strings():
    lib = _nkb.lib()
    assert lib.nkb_status_str(0) == b"ok"
    assert lib.nkb_status_str(3) == b"plan error"


def test_device_count_is_callable():
    n = ctypes.c_int(-1)
    assert _nkb.lib().nkb_device_count(ctypes.byref(n)) == 0
    assert n.value >= 0


def test_calls_before_init_fail_cleanly():
    lib = _nkb.lib()
    n = ctypes.c_int()
    if lib.nkb_device_count(ctypes.byref(n)) == 0 and n.value > 0:
        pytest.skip("a GPU is visible; the uninitialised state is not reachable here")
    h = ctypes.c_void_p()
    st = lib.nkb_alloc(16, 0, ctypes.byref(h))
    assert st == 6  # NKB_ERR_STATE
    assert b"not initialised" in lib.nkb_last_error()
    st = lib.nkb_init(0)
    assert st != 0 and lib.nkb_last_error()
    with pytest.raises(_nkb.NkbError):
        _nkb.call("nkb_synchronize")


def test_null_arguments_rejected():
    lib = _nkb.lib()
    assert lib.nkb_device_count(None) == 1
    assert lib.nkb_plan_num_io(None, None, None) == 1


def test_wait_limit_setting():
    lib = _nkb.lib()
    old = ctypes.c_uint64()
    assert lib.nkb_get_wait_limit_us(ctypes.byref(old)) == 0 and old.value > 0
    try:
        assert lib.nkb_set_wait_limit_us(5000) == 0
        v = ctypes.c_uint64()
        lib.nkb_get_wait_limit_us(ctypes.byref(v))
        assert v.value == 5000
        assert lib.nkb_set_wait_limit_us(0) == 1 and b"positive" in lib.nkb_last_error()
        assert lib.nkb_get_wait_limit_us(None) == 1
    finally:
        lib.nkb_set_wait_limit_us(old.value)
