"""Pipelined execution: the copies of one step overlap the compute of another.

The reference executes a loaded model synchronously (``spike_model.py:192-268``:
write the inputs, execute, read the outputs); a loop of such calls leaves the
GPU idle during every host<->device copy.  ``run_pipelined`` keeps the same
per-step semantics -- each step uploads its inputs from host memory, runs the
plan and reads its outputs back to host memory -- but issues the three on
separate streams with two device buffer sets, so step i+1's upload and step
i-1's read-back run while step i computes (host memory must be page-locked for
the copies to be asynchronous).  Under tensor parallelism with ``split``, each
rank uploads only its 1/world of every step input's rows and an in-place
all-gather over NVLink completes the input on every rank before the execute;
each rank reads back its 1/world of every fetched output's rows.
"""

import ctypes
from typing import Dict, Optional, Sequence, Union

import numpy as np

from nkipy_b200.spike import _nkb
from nkipy_b200.spike._nkb import SpikeError


def _host_ptr(arr: np.ndarray):
    if not isinstance(arr, np.ndarray) or not arr.flags.c_contiguous:
        raise SpikeError("pipelined host buffers must be C-contiguous numpy arrays")
    return ctypes.c_void_p(arr.ctypes.data), arr.nbytes


class _Resources:
    """Three streams and per-slot events, created once per model."""

    def __init__(self):
        self.h2d, self.comp, self.d2h = (self._stream() for _ in range(3))
        self.up = [self._event() for _ in range(2)]
        self.done = [self._event() for _ in range(2)]
        self.down = [self._event() for _ in range(2)]

    @staticmethod
    def _stream():
        s = ctypes.c_void_p()
        _nkb.call("nkb_stream_create", ctypes.byref(s))
        return s

    @staticmethod
    def _event():
        e = ctypes.c_void_p()
        _nkb.call("nkb_event_create", ctypes.byref(e))
        return e

    def __del__(self):
        if getattr(_nkb, "_lib", None) is None:
            return
        try:
            for e in self.up + self.done + self.down:
                _nkb.lib().nkb_event_destroy(e)
            for s in (self.h2d, self.comp, self.d2h):
                _nkb.lib().nkb_stream_destroy(s)
        except Exception:
            pass


def run_pipelined(spike, model, resident: Dict[str, object], host_inputs: Dict[str, Union[np.ndarray, Sequence[np.ndarray]]],
                  host_outputs: Dict[str, np.ndarray], steps: int, split: bool = False,
                  bind: Optional[Dict[str, object]] = None, use_graph: bool = True, state: Optional[dict] = None):
    """Run ``steps`` executes of ``model`` (an ``NkbModel``) with overlapped copies.

    ``resident``: input name -> ``NkbTensor`` that stays on the device (weights).
    ``host_inputs``: input name -> page-locked host array uploaded every step, or a
    sequence of arrays (step i uses element i % len).  ``host_outputs``: output name
    -> page-locked host array that receives every step's result (the last one stays).
    ``bind``: output name -> ``NkbTensor`` an output is bound to (a mutated input's
    in-place output); the other outputs get a device buffer per slot.  ``split``:
    tensor-parallel row split (see the module docstring).  ``state``: a dict kept by
    the caller across calls, holding the device buffers, streams and events.
    Returns after the last read-back completed; raises ``NkbError`` when a kernel
    reported a device error."""
    io = model.io
    in_specs = {s["name"]: s for s in io["inputs"]}
    out_specs = {s["name"]: s for s in io["outputs"]}
    step_names = list(host_inputs)
    missing = set(in_specs) - set(resident) - set(step_names)
    if missing:
        raise SpikeError(f"inputs neither resident nor fed per step: {sorted(missing)}")
    bind = bind or {}
    world, rank = (model.world_size, model.rank_id) if split else (1, 0)
    if split and model.comm is None:
        raise SpikeError("a row split needs a plan loaded with collectives (cc_enabled)")
    state = state if state is not None else {}
    if "res" not in state:
        state["res"] = _Resources()
        state["bufs"] = {}
    res = state["res"]

    def slot_buf(kind, name, slot, nbytes):
        key = (kind, name, slot)
        t = state["bufs"].get(key)
        if t is None or t.size != nbytes:
            t = spike.allocate_tensor(nbytes, name=f"{name}.slot{slot}")
            state["bufs"][key] = t
        return t

    def nbytes_of(spec):
        dt = np.dtype(spec["dtype"]) if spec["dtype"] != "bfloat16" else np.dtype(np.uint16)
        return max(1, int(np.prod(spec["shape"], dtype=np.int64)) * dt.itemsize)

    feeds = {n: (v if isinstance(v, (list, tuple)) else [v]) for n, v in host_inputs.items()}
    for n, arrs in feeds.items():
        for a in arrs:
            _, nb = _host_ptr(a)
            if nb * world != nbytes_of(in_specs[n]):
                raise SpikeError(f"host input {n!r}: {nb} bytes, plan wants {nbytes_of(in_specs[n])} / {world}")
    for n, a in host_outputs.items():
        _, nb = _host_ptr(a)
        if nb * world != nbytes_of(out_specs[n]):
            raise SpikeError(f"host output {n!r}: {nb} bytes, plan wants {nbytes_of(out_specs[n])} / {world}")

    handles = []
    for slot in range(2):
        ins = {n: resident[n] for n in resident}
        for n in step_names:
            ins[n] = slot_buf("in", n, slot, nbytes_of(in_specs[n]))
        outs = {}
        for n, spec in out_specs.items():
            outs[n] = bind[n] if n in bind else slot_buf("out", n, slot, nbytes_of(spec))
        handles.append((ins, outs, spike._io_lists(model, ins, outs)))

    for i in range(steps):
        slot = i % 2
        ins, outs, (I, ni, O, no) = handles[slot]
        if i >= 2:  # the slot's previous execute has finished reading its inputs
            _nkb.call("nkb_stream_wait_event", res.h2d, res.done[slot])
        for n in step_names:
            src, nb = _host_ptr(feeds[n][i % len(feeds[n])])
            _nkb.call("nkb_h2d_async", ins[n].handle, src, nb, rank * nb, res.h2d)
        _nkb.call("nkb_event_record", res.up[slot], res.h2d)
        _nkb.call("nkb_stream_wait_event", res.comp, res.up[slot])
        if i >= 2:  # the slot's previous read-back has finished with its outputs
            _nkb.call("nkb_stream_wait_event", res.comp, res.down[slot])
        if split:
            for n in step_names:
                nb = ins[n].size // world
                base = ins[n].va
                _nkb.call("nkb_comm_all_gather", model.comm, ctypes.c_void_p(base + rank * nb), ctypes.c_void_p(base),
                          nb, 6, res.comp)  # 6: NKB_U8
        _nkb.call("nkb_execute", model.handle, I, ni, O, no, res.comp, int(use_graph))
        _nkb.call("nkb_event_record", res.done[slot], res.comp)
        _nkb.call("nkb_stream_wait_event", res.d2h, res.done[slot])
        for n, a in host_outputs.items():
            dst, nb = _host_ptr(a)
            _nkb.call("nkb_d2h_async", outs[n].handle, dst, nb, rank * nb, res.d2h)
        _nkb.call("nkb_event_record", res.down[slot], res.d2h)
    for s in (res.h2d, res.comp, res.d2h):
        _nkb.call("nkb_stream_synchronize", s)
    flag = ctypes.c_int()
    _nkb.call("nkb_device_error", ctypes.byref(flag))
    if flag.value:
        raise _nkb.NkbError(7, "a kernel's bounded wait expired; results are invalid")
    return handles[(steps - 1) % 2][1] if steps else None
