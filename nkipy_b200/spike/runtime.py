"""The ``Spike`` runtime object over libnkb (reference: ``spike/src/spike.cpp``,
``spike/src/include/spike.h:28-86``, nanobind surface ``python_bindings.cpp``).

Same method names and meanings as the reference's ``_spike.Spike``:
``allocate_tensor`` / ``slice_from_tensor`` / ``free_tensor``,
``tensor_write`` / ``tensor_read`` (+ ``_pybuffer`` variants, bounds-checked),
``load_model`` / ``unload_model``, ``execute`` (name-keyed tensor dicts) and
``get_tensor_info``.  A "model" is a launch plan file (``*.nkbplan``) instead
of a NEFF; ``core_id`` is the CUDA device of this process.  One runtime per
process, bound to one GPU (``NKB_DEVICE``, else ``LOCAL_RANK``, else 0).
"""

import ctypes
import json
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np

from nkipy_b200.spike import _nkb
from nkipy_b200.spike._nkb import NkbError, SpikeError

COMM_ID_BYTES = 128


def default_device() -> int:
    for var in ("NKB_DEVICE", "LOCAL_RANK"):
        v = os.environ.get(var)
        if v is not None and v.strip().isdigit():
            return int(v)
    return 0


@dataclass
class TensorMetadata:
    size: int
    dtype: str
    shape: List[int]


@dataclass
class ModelTensorInfo:
    inputs: Dict[str, TensorMetadata] = field(default_factory=dict)
    outputs: Dict[str, TensorMetadata] = field(default_factory=dict)


class NkbTensor:
    """A device buffer handle (reference ``NrtTensor``, tensor.h:14-53)."""

    __slots__ = ("handle", "size", "core_id", "name", "_freed", "_keepalive", "__weakref__")

    def __init__(self, handle, size, core_id, name=None, keepalive=None):
        self.handle = handle
        self.size = size
        self.core_id = core_id
        self.name = name
        self._freed = False
        self._keepalive = keepalive

    @property
    def va(self) -> int:
        ptr = ctypes.c_void_p()
        _nkb.call("nkb_buf_info", self.handle, None, None, ctypes.byref(ptr))
        return ptr.value or 0

    def __del__(self):
        if not self._freed and self.handle and getattr(_nkb, "_lib", None) is not None:
            try:
                _nkb.lib().nkb_free(self.handle)
            except Exception:
                pass
            self._freed = True

    def __repr__(self):
        return f"NkbTensor(name={self.name}, size={self.size}, core_id={self.core_id})"


class NkbModel:
    """A loaded launch plan (reference ``NrtModel``, model.h:12-55)."""

    def __init__(self, handle, core_id, path, io, rank_id=0, world_size=1, comm=None):
        self.handle = handle
        self.core_id = core_id
        self.path = path
        self.io = io
        self.rank_id = rank_id
        self.world_size = world_size
        self.comm = comm
        self.symmetric = False  # all-reduces run inside NVSwitch (bound symmetric region)
        self.last_trace = None  # path of the last execute's trace (save_trace=True)
        n = ctypes.c_int()
        _nkb.call("nkb_plan_num_launches", handle, ctypes.byref(n))
        self.num_launches = n.value
        s = ctypes.c_size_t()
        _nkb.call("nkb_plan_scratch_bytes", handle, ctypes.byref(s))
        self.scratch_bytes = s.value

    @property
    def graph_kernels(self) -> int:
        """Kernels one graph-replayed execute launches (the kernel nodes of the
        plan's last captured CUDA graph; -1 before the first one)."""
        n = ctypes.c_int()
        _nkb.call("nkb_plan_graph_kernels", self.handle, ctypes.byref(n))
        return n.value

    def __del__(self):
        if self.handle and getattr(_nkb, "_lib", None) is not None:
            try:
                _nkb.lib().nkb_plan_free(self.handle)
            except Exception:
                pass
            self.handle = None

    def __repr__(self):
        return f"NkbModel({os.path.basename(self.path)}, core_id={self.core_id}, launches={self.num_launches})"


_COMMS = {}


def _communicator(rank: int, world: int, device: int):
    """One NCCL communicator per (world, rank) and process.

    The unique id is created on rank 0 and broadcast with torch.distributed --
    the same control plane the reference uses to distribute its NEFF path
    (runtime/device_kernel.py:142-197).
    """
    key = (world, rank)
    if key in _COMMS:
        return _COMMS[key]
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        raise ValueError("a collective plan needs torch.distributed to be initialised to exchange the NCCL id")
    buf = (ctypes.c_uint8 * COMM_ID_BYTES)()
    if rank == 0:
        _nkb.call("nkb_comm_unique_id", ctypes.cast(buf, ctypes.c_void_p))
    obj = [bytes(buf)]
    dist.broadcast_object_list(obj, src=0)
    ctypes.memmove(buf, obj[0], COMM_ID_BYTES)
    comm = ctypes.c_void_p()
    _nkb.call("nkb_comm_init", ctypes.cast(buf, ctypes.c_void_p), rank, world, device, ctypes.byref(comm))
    _COMMS[key] = comm
    return comm


_SYMM: Dict[tuple, list] = {}  # (world, rank) -> [capacity bytes, tensors kept alive]


def _symm_bytes(plan_text: str) -> int:
    """Bytes of the symmetric region a plan's all-reduce operands need (its "symm" line)."""
    for line in plan_text.splitlines():
        if line.startswith("symm "):
            return int(line.split()[1])
        if line.startswith("steps "):
            break
    return 0


def _bind_symmetric(comm, rank: int, world: int, device: int, need: int) -> bool:
    """Give the communicator a symmetric region for all-reduces inside NVSwitch.

    The region is a PyTorch symmetric-memory allocation (every rank maps every
    other rank's copy, plus an NVLink multicast object over all of them); all
    ranks take the same decision, and a rank without multicast support makes
    every rank keep NCCL.  NKB_SYMM: "auto" (default) and "force" bind it at
    any world size ("force" fails loudly when it cannot); "0" never.  With a
    region bound, a row-parallel GEMM reduces its output inside its own kernel
    (multimem through NVSwitch) while its later tiles compute, which beats the
    GEMM followed by NCCL's all-reduce from 2 ranks up on B200.  Regions are
    never freed: plans captured into CUDA graphs keep their addresses.
    """
    mode = os.environ.get("NKB_SYMM", "auto")
    if need <= 0 or mode == "0":
        return False
    entry = _SYMM.get((world, rank))
    if entry is not None and entry[0] >= need:
        return True
    import torch
    import torch.distributed as dist
    import torch.distributed._symmetric_memory as symm_mem

    flag = int(_nkb.lib().nkb_comm_symm_flag_bytes())
    cap = max(need, 64 << 20)
    nbytes = cap + flag
    t = symm_mem.empty(nbytes, dtype=torch.uint8, device=torch.device("cuda", device))
    h = symm_mem.rendezvous(t, dist.group.WORLD)
    peers = [int(x) for x in h.buffer_ptrs]
    ok = int(h.multicast_ptr) != 0 and len(peers) == world and peers[rank] == t.data_ptr()
    votes = [None] * world
    dist.all_gather_object(votes, bool(ok))
    if not all(votes):
        return False
    arr = (ctypes.c_void_p * world)(*peers)
    _nkb.call("nkb_comm_bind_symm", comm, t.data_ptr(), int(h.multicast_ptr), arr, world, nbytes)
    torch.cuda.synchronize(device)
    dist.barrier()
    kept = (entry[1] if entry else []) + [t, h]
    _SYMM[(world, rank)] = [cap, kept]
    return True


class Spike:
    def __init__(self, verbose: int = 0, device: Optional[int] = None):
        self.verbose = verbose
        self.device = default_device() if device is None else device
        _nkb.call("nkb_init", self.device)
        self._closed = False

    @staticmethod
    def get_visible_neuron_core_count() -> int:
        """Number of visible CUDA devices (name kept from the reference)."""
        try:
            n = ctypes.c_int()
            _nkb.call("nkb_device_count", ctypes.byref(n))
            return n.value
        except (ImportError, NkbError, OSError):
            return 0

    get_visible_device_count = get_visible_neuron_core_count

    def close(self) -> int:
        if not self._closed:
            for c in list(_COMMS.values()):
                _nkb.lib().nkb_comm_free(c)
            _COMMS.clear()
            _nkb.call("nkb_shutdown")
            self._closed = True
        return 0

    def is_closed(self) -> bool:
        return self._closed

    def _check_core(self, core_id):
        if core_id != self.device:
            raise SpikeError(f"core_id {core_id} is not this process's device {self.device}")

    # -- tensors --------------------------------------------------------------
    def allocate_tensor(self, size: int, core_id: Optional[int] = None, name: Optional[str] = None) -> NkbTensor:
        core_id = self.device if core_id is None else core_id
        self._check_core(core_id)
        h = ctypes.c_void_p()
        _nkb.call("nkb_alloc", int(size), core_id, ctypes.byref(h))
        return NkbTensor(h, int(size), core_id, name)

    def wrap_device_memory(self, ptr: int, size: int, name=None, keepalive=None) -> NkbTensor:
        h = ctypes.c_void_p()
        _nkb.call("nkb_wrap", ctypes.c_void_p(ptr), int(size), self.device, ctypes.byref(h))
        return NkbTensor(h, int(size), self.device, name, keepalive=keepalive)

    def slice_from_tensor(self, source: NkbTensor, offset: int = 0, size: int = 0, name: Optional[str] = None):
        self._live(source)
        h = ctypes.c_void_p()
        _nkb.call("nkb_slice", source.handle, int(offset), int(size), ctypes.byref(h))
        real = size if size else source.size - offset
        return NkbTensor(h, int(real), source.core_id, name, keepalive=source)

    def free_tensor(self, tensor: NkbTensor):
        self._live(tensor)
        _nkb.call("nkb_free", tensor.handle)
        tensor._freed = True

    @staticmethod
    def _live(t: NkbTensor):
        if t._freed:
            raise SpikeError(f"tensor {t.name!r} has been freed")

    def tensor_write(self, tensor: NkbTensor, data: bytes, offset: int = 0):
        self._live(tensor)
        buf = ctypes.create_string_buffer(bytes(data), len(data))
        _nkb.call("nkb_h2d", tensor.handle, ctypes.cast(buf, ctypes.c_void_p), len(data), int(offset))

    def tensor_read(self, tensor: NkbTensor, offset: int = 0, size: int = 0) -> bytes:
        self._live(tensor)
        size = size or tensor.size - offset
        buf = ctypes.create_string_buffer(size)
        _nkb.call("nkb_d2h", tensor.handle, ctypes.cast(buf, ctypes.c_void_p), int(size), int(offset))
        return buf.raw

    @staticmethod
    def _bytes_view(data):
        """A uint8 ndarray over ``data`` (ndarrays of any dtype, incl. bf16, or buffers)."""
        if isinstance(data, np.ndarray):
            if not data.flags.c_contiguous:
                raise SpikeError("buffer must be C-contiguous")
            return data.reshape(-1).view(np.uint8)
        return np.frombuffer(memoryview(data).cast("B"), dtype=np.uint8)

    def tensor_write_from_pybuffer(self, tensor: NkbTensor, data, offset: int = 0):
        self._live(tensor)
        arr = self._bytes_view(np.ascontiguousarray(data) if isinstance(data, np.ndarray) else data)
        _nkb.call("nkb_h2d", tensor.handle, arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes, int(offset))

    def tensor_read_to_pybuffer(self, tensor: NkbTensor, data, offset: int = 0):
        self._live(tensor)
        arr = self._bytes_view(data)
        if not arr.flags.writeable:
            raise SpikeError("destination buffer is read-only")
        _nkb.call("nkb_d2h", tensor.handle, arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes, int(offset))

    # -- models -------------------------------------------------------------------
    def load_model(self, plan_file: str, core_id: Optional[int] = None, cc_enabled: bool = False,
                   rank_id: int = 0, world_size: int = 1) -> NkbModel:
        core_id = self.device if core_id is None else core_id
        self._check_core(core_id)
        text, consts, io = read_plan_files(plan_file)
        h = ctypes.c_void_p()
        raw = text.encode()
        _nkb.call("nkb_plan_load", raw, len(raw), core_id, ctypes.byref(h))
        model = NkbModel(h, core_id, plan_file, io, rank_id, world_size)
        for i, c in enumerate(consts):
            c = np.ascontiguousarray(c)
            _nkb.call("nkb_plan_set_const", h, i, c.ctypes.data_as(ctypes.c_void_p), c.nbytes)
        if cc_enabled and world_size > 1:
            model.comm = _communicator(rank_id, world_size, core_id)
            _nkb.call("nkb_plan_bind_comm", h, model.comm)
            model.symmetric = _bind_symmetric(model.comm, rank_id, world_size, core_id, _symm_bytes(text))
        elif io.get("needs_comm"):
            raise ValueError("this plan contains collectives: load it with cc_enabled=True, rank_id and world_size")
        return model

    def unload_model(self, model: NkbModel):
        if model.handle:
            _nkb.call("nkb_plan_free", model.handle)
            model.handle = None

    def _io_lists(self, model, inputs, outputs):
        ins, outs = [], []
        for spec in model.io["inputs"]:
            t = inputs.get(spec["name"])
            if t is None:
                raise SpikeError(f"missing input '{spec['name']}'")
            self._live(t)
            ins.append(t.handle)
        for spec in model.io["outputs"]:
            t = outputs.get(spec["name"])
            if t is None:
                raise SpikeError(f"missing output '{spec['name']}'")
            self._live(t)
            outs.append(t.handle)
        extra = set(inputs) - {s["name"] for s in model.io["inputs"]}
        if extra:
            raise SpikeError(f"unknown inputs {sorted(extra)}")
        extra = set(outputs) - {s["name"] for s in model.io["outputs"]}
        if extra:
            raise SpikeError(f"unknown outputs {sorted(extra)}")
        I = (ctypes.c_void_p * max(1, len(ins)))(*[h.value for h in ins])
        O = (ctypes.c_void_p * max(1, len(outs)))(*[h.value for h in outs])
        return I, len(ins), O, len(outs)

    def execute(self, model: NkbModel, inputs: Dict[str, NkbTensor], outputs: Dict[str, NkbTensor],
                ntff_name: Optional[str] = None, save_trace: bool = False, use_graph: bool = False):
        I, ni, O, no = self._io_lists(model, inputs, outputs)
        if save_trace:
            # the reference writes a device profile of this execute (an NTFF file named
            # ntff_name); here: a Chrome-trace JSON of the execute's launches
            n = max(1, model.num_launches)
            start, dur = (ctypes.c_float * n)(), (ctypes.c_float * n)()
            _nkb.call("nkb_trace_execute", model.handle, I, ni, O, no, start, dur)
            model.last_trace = write_trace(model, [float(x) for x in start[: model.num_launches]],
                                           [float(x) for x in dur[: model.num_launches]], ntff_name)
        else:
            _nkb.call("nkb_execute", model.handle, I, ni, O, no, None, int(use_graph))
        _nkb.call("nkb_synchronize")
        flag = ctypes.c_int()
        _nkb.call("nkb_device_error", ctypes.byref(flag))
        if flag.value:
            raise NkbError(7, "a kernel's bounded wait expired; results are invalid")

    def all_gather_in_place(self, model: NkbModel, tensor: NkbTensor, bytes_per_rank: int, offset: int = 0):
        """All-gather over the model's communicator, in place in ``tensor``:
        rank r contributes the ``bytes_per_rank`` bytes at ``offset + r *
        bytes_per_rank`` and every rank ends with all ``world`` blocks (the
        reference's ``all_gather`` collective, ``core/ops/collectives.py:34-53``,
        issued outside a plan).  Ordered with the runtime's other work on its
        stream; bounds-checked against the tensor."""
        self._live(tensor)
        if model.comm is None or model.world_size <= 1:
            return
        n, world = int(bytes_per_rank), model.world_size
        if offset < 0 or n < 0 or offset + n * world > tensor.size:
            raise SpikeError(f"all-gather of {world} x {n} bytes at offset {offset} exceeds tensor of {tensor.size} bytes")
        base = tensor.va + int(offset)
        _nkb.call("nkb_comm_all_gather", model.comm, ctypes.c_void_p(base + model.rank_id * n), ctypes.c_void_p(base),
                  n, 6, None)  # 6: NKB_U8

    def time_execute(self, model: NkbModel, inputs, outputs, warmup: int, iters: int, use_graph: bool = True):
        I, ni, O, no = self._io_lists(model, inputs, outputs)
        ms = (ctypes.c_float * iters)()
        _nkb.call("nkb_time_execute", model.handle, I, ni, O, no, warmup, iters, int(use_graph), ms)
        return [float(v) for v in ms]

    def time_execute_steps(self, model: NkbModel, inputs, outputs):
        """One graph replay with an event between every two launches: (the
        execute's device time, [each launch's time inside it]) in ms."""
        I, ni, O, no = self._io_lists(model, inputs, outputs)
        total = ctypes.c_float()
        ms = (ctypes.c_float * max(1, model.num_launches))()
        _nkb.call("nkb_time_execute_steps", model.handle, I, ni, O, no, ctypes.byref(total), ms)
        return float(total.value), [float(ms[i]) for i in range(model.num_launches)]

    def time_steps(self, model: NkbModel, inputs, outputs, iters: int):
        """Mean device time of every launch of the plan (ms), in plan order."""
        I, ni, O, no = self._io_lists(model, inputs, outputs)
        ms = (ctypes.c_float * max(1, model.num_launches))()
        _nkb.call("nkb_time_steps", model.handle, I, ni, O, no, iters, ms)
        return [float(ms[i]) for i in range(model.num_launches)]

    def get_tensor_info(self, model: NkbModel) -> ModelTensorInfo:
        info = ModelTensorInfo()
        for key, dst in (("inputs", info.inputs), ("outputs", info.outputs)):
            for spec in model.io[key]:
                dt = np.dtype(spec["dtype"]) if spec["dtype"] != "bfloat16" else None
                size = int(np.prod(spec["shape"], dtype=np.int64)) * (2 if dt is None else dt.itemsize)
                dst[spec["name"]] = TensorMetadata(size=size, dtype=spec["dtype"], shape=list(spec["shape"]))
        return info


def write_trace(model, start_ms, dur_ms, path=None) -> str:
    """Chrome-trace JSON (chrome://tracing, Perfetto) of one execute: an event per
    launch, named after its kernel, on the device's timeline.  ``path`` defaults
    to ``<plan>.trace.json``; a name without a directory goes next to the plan."""
    kernels = []
    with open(model.path) as f:
        for line in f:
            if line.startswith("step "):
                kernels.append(line.split()[1])
    events = [{"name": k, "cat": "kernel", "ph": "X", "ts": s * 1e3, "dur": d * 1e3, "pid": model.core_id,
               "tid": 0, "args": {"launch": i}} for i, (k, s, d) in enumerate(zip(kernels, start_ms, dur_ms))]
    if not path:
        path = model.path + ".trace.json"
    elif not os.path.dirname(path):
        path = os.path.join(os.path.dirname(model.path), path)
    with open(path, "w") as f:
        json.dump({"traceEvents": events, "displayTimeUnit": "ms"}, f)
    return path


# -- plan files ---------------------------------------------------------------------
def write_plan_files(plan, path: str):
    """``<path>`` (plan text), ``<path>.consts.npz`` and ``<path>.io.json``."""
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        f.write(plan.to_text())
    np.savez(path + ".consts.npz", **{f"c{i}": c.view(np.uint8).reshape(-1) for i, c in enumerate(plan.consts)})
    io = {
        "name": plan.name,
        "inputs": [{"name": s.name, "shape": list(s.shape), "dtype": str(np.dtype(s.dtype))} for s in plan.inputs],
        "outputs": [{"name": s.name, "shape": list(s.shape), "dtype": str(np.dtype(s.dtype))} for s in plan.outputs],
        "aliases": plan.aliases,
        "needs_comm": plan.needs_comm,
        "launches": len(plan.steps),
        "kernels": plan.kernel_counts(),
    }
    with open(path + ".io.json", "w") as f:
        json.dump(io, f, indent=1)


def read_plan_files(path: str):
    if not os.path.exists(path):
        raise FileNotFoundError(f"plan file not found: {path}")
    with open(path) as f:
        text = f.read()
    with open(path + ".io.json") as f:
        io = json.load(f)
    consts = []
    cpath = path + ".consts.npz"
    if os.path.exists(cpath):
        with np.load(cpath) as z:
            consts = [z[f"c{i}"] for i in range(len(z.files))]
    return text, consts, io
