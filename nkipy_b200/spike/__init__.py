"""Spike-equivalent Python layer over libnkb.

Mirrors the reference package ``spike`` (spike/src/spike/*.py):
``SpikeTensor`` (from_numpy / numpy / write_from_numpy), ``SpikeModel``
(load / __call__ with name-keyed tensors / benchmark), ``BenchmarkResult``,
and the thread-safe runtime singleton (``configure`` / ``reset`` /
``get_spike_singleton``).
"""

import atexit
import math
import os
import threading
import time
import warnings
from dataclasses import dataclass, field
from pathlib import Path
from typing import Dict, Iterable, List, Optional

import ml_dtypes
import numpy as np

from nkipy_b200.spike._nkb import NkbError, NrtError, SpikeError, SpikeRuntimeError  # noqa: F401
from nkipy_b200.spike.runtime import ModelTensorInfo, NkbModel, NkbTensor, Spike, TensorMetadata  # noqa: F401

_runtime: Optional[Spike] = None
_lock = threading.Lock()


def configure(visible_cores: Optional[Iterable[int]] = None) -> None:
    """Select the device before the runtime starts (reference spike_singleton.py:59-90).

    ``visible_cores`` names CUDA devices; the first one becomes this
    process's device.
    """
    with _lock:
        if _runtime is not None:
            raise RuntimeError("Cannot configure: runtime is already active. Call reset() first.")
    if visible_cores is None:
        return
    if isinstance(visible_cores, int):
        raise TypeError(f"visible_cores must be an iterable, not int. Use [{visible_cores}]")
    cores = list(visible_cores)
    for c in cores:
        if not isinstance(c, int):
            raise TypeError(f"visible_cores must contain integers, got {type(c)}: {c}")
        if c < 0:
            raise ValueError(f"Core ID must be non-negative, got {c}")
    if cores:
        os.environ["NKB_DEVICE"] = str(cores[0])


def reset() -> None:
    global _runtime
    with _lock:
        if _runtime is not None:
            warnings.warn("spike.reset() called: existing tensors and models are invalid.", UserWarning, stacklevel=2)
            _runtime.close()
            _runtime = None


def get_spike_singleton() -> Spike:
    global _runtime
    if _runtime is not None:
        return _runtime
    with _lock:
        if _runtime is None:
            _runtime = Spike()
        return _runtime


@atexit.register
def _cleanup():
    global _runtime
    _runtime = None


@dataclass
class BenchmarkResult:
    """Same fields as the reference (spike_model.py:20-39)."""

    mean_ms: float
    min_ms: float
    max_ms: float
    std_dev_ms: float
    iterations: int
    warmup_iterations: int
    durations_ms: List[float] = field(default_factory=list)

    def __repr__(self):
        return (
            f"BenchmarkResult(mean={self.mean_ms:.4f}ms, min={self.min_ms:.4f}ms, max={self.max_ms:.4f}ms, "
            f"std_dev={self.std_dev_ms:.4f}ms, iterations={self.iterations}, warmup_iterations={self.warmup_iterations})"
        )


def _result(d, warmup):
    n = len(d)
    mean = sum(d) / n
    return BenchmarkResult(mean, min(d), max(d), math.sqrt(sum((x - mean) ** 2 for x in d) / n), n, warmup, list(d))


def _np_dtype(name):
    return np.dtype(ml_dtypes.bfloat16) if name == "bfloat16" else np.dtype(name)


class SpikeTensor:
    def __init__(self, tensor_ref: NkbTensor, shape, dtype, name: str = None):
        self.tensor_ref = tensor_ref
        self.shape = (shape,) if isinstance(shape, int) else tuple(shape)
        self.dtype = np.dtype(dtype)
        self.name = name

    @classmethod
    def from_numpy(cls, array: np.ndarray, name: str = None, core_id=None):
        array = np.ascontiguousarray(array)
        spike = get_spike_singleton()
        ref = spike.allocate_tensor(size=max(1, array.nbytes), core_id=core_id, name=name)
        if array.nbytes:
            spike.tensor_write_from_pybuffer(ref, array)
        return cls(ref, array.shape, array.dtype, name)

    @classmethod
    def empty(cls, shape, dtype, name=None, core_id=None):
        nbytes = int(np.prod(shape, dtype=np.int64)) * np.dtype(dtype).itemsize
        ref = get_spike_singleton().allocate_tensor(size=max(1, nbytes), core_id=core_id, name=name)
        return cls(ref, shape, dtype, name)

    def numpy(self) -> np.ndarray:
        out = np.empty(self.shape, dtype=self.dtype)
        if out.nbytes:
            get_spike_singleton().tensor_read_to_pybuffer(self.tensor_ref, out)
        return out

    def write_from_numpy(self, array: np.ndarray):
        array = np.ascontiguousarray(array)
        expected = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        if array.nbytes != expected:
            raise ValueError(f"Size mismatch: source {array.nbytes} bytes, target {expected} bytes")
        get_spike_singleton().tensor_write_from_pybuffer(self.tensor_ref, array)

    def __repr__(self):
        return f"{self.__class__.__name__}(shape={self.shape}, dtype={self.dtype}, name={self.name})"


class SpikeModel:
    """A loaded launch plan with name-keyed execution (reference spike_model.py:102-343)."""

    def __init__(self, model_ref: NkbModel, name: str, neff_path):
        self.model_ref = model_ref
        self.name = name
        self.neff_path = Path(neff_path)
        info = get_spike_singleton().get_tensor_info(model_ref)
        self.input_tensors_info = info.inputs
        self.output_tensors_info = info.outputs

    @property
    def plan_path(self):
        return self.neff_path

    @classmethod
    def load_from_neff(cls, neff_path, name=None, core_id=None, cc_enabled=False, rank_id=0, world_size=1):
        """Load a plan file (the reference name is kept: the plan replaces the NEFF)."""
        path = Path(neff_path)
        name = name or path.stem
        ref = get_spike_singleton().load_model(str(path), core_id, cc_enabled, rank_id, world_size)
        return cls(ref, name, path)

    load_from_plan = load_from_neff

    def allocate_output_tensors(self) -> List[SpikeTensor]:
        out = []
        for k, v in self.output_tensors_info.items():
            dt = _np_dtype(v.dtype)
            t = SpikeTensor.empty(tuple(v.shape), dt, name=k, core_id=self.model_ref.core_id)
            assert t.tensor_ref.size == max(1, v.size), f"Size mismatch for {k}"
            out.append(t)
        return out

    def _validate_io(self, inputs, outputs):
        core = self.model_ref.core_id
        for kind, given, info in (("Input", inputs, self.input_tensors_info), ("Output", outputs, self.output_tensors_info)):
            for k, v in given.items():
                assert k in info, f"{kind} {k}: not a {kind.lower()} of this kernel (expected {sorted(info)})"
                assert v.tensor_ref.core_id == core, (
                    f"{kind} {k}: expected model and tensor on the same core, got model core_id {core} and tensor "
                    f"core_id {v.tensor_ref.core_id}"
                )
                assert tuple(v.shape) == tuple(info[k].shape), f"{kind} {k}: expected shape {tuple(info[k].shape)}, got {v.shape}"
                assert v.dtype == _np_dtype(info[k].dtype), f"{kind} {k}: expected dtype {info[k].dtype}, got {v.dtype}"

    def __call__(self, inputs: Dict[str, SpikeTensor], outputs: Dict[str, SpikeTensor] = None, save_trace=False,
                 ntff_name=None, use_graph=False):
        auto = outputs is None
        if auto:
            outputs = {t.name: t for t in self.allocate_output_tensors()}
        self._validate_io(inputs, outputs)
        get_spike_singleton().execute(
            self.model_ref,
            {k: v.tensor_ref for k, v in inputs.items()},
            {k: v.tensor_ref for k, v in outputs.items()},
            ntff_name=ntff_name,
            save_trace=save_trace,
            use_graph=use_graph,
        )
        if auto:
            return outputs

    def run_steps(self, resident: Dict[str, SpikeTensor], host_inputs, host_outputs, steps: int, split: bool = False,
                  bind: Dict[str, SpikeTensor] = None, use_graph: bool = True):
        """Run ``steps`` executes with each step's copies overlapping other steps'
        compute (``nkipy_b200.spike.pipeline.run_pipelined``): ``resident`` device
        inputs stay, ``host_inputs`` (name -> page-locked array, or a sequence of
        them, one per step) are uploaded every step, ``host_outputs`` (name ->
        page-locked array) receive every step's result; ``bind`` fixes outputs to
        tensors (a mutated input's in-place output); ``split`` uploads and reads
        back this rank's rows only, the inputs completed by an all-gather.
        Device buffers, streams and events are kept on the model for the next call."""
        from nkipy_b200.spike.pipeline import run_pipelined

        self._validate_io(resident, bind or {})
        state = self.__dict__.setdefault("_pipeline_state", {})
        return run_pipelined(get_spike_singleton(), self.model_ref, {k: v.tensor_ref for k, v in resident.items()},
                             host_inputs, host_outputs, steps, split=split,
                             bind={k: v.tensor_ref for k, v in (bind or {}).items()}, use_graph=use_graph, state=state)

    def benchmark(self, inputs, outputs=None, warmup_iter=5, benchmark_iter=5, mode: str = "device"):
        """'device': CUDA-event time per execute; 'host': wall clock per synchronous execute."""
        if mode not in ("device", "host"):
            raise ValueError(f"Invalid benchmark mode '{mode}'. Use 'device' or 'host'.")
        if outputs is None:
            outputs = {t.name: t for t in self.allocate_output_tensors()}
        self._validate_io(inputs, outputs)
        spike = get_spike_singleton()
        ins = {k: v.tensor_ref for k, v in inputs.items()}
        outs = {k: v.tensor_ref for k, v in outputs.items()}
        if mode == "device":
            d = spike.time_execute(self.model_ref, ins, outs, warmup_iter, benchmark_iter)
            return _result(d, warmup_iter)
        for _ in range(warmup_iter):
            spike.execute(self.model_ref, ins, outs)
        d = []
        for _ in range(benchmark_iter):
            t0 = time.perf_counter()
            spike.execute(self.model_ref, ins, outs)
            d.append((time.perf_counter() - t0) * 1000.0)
        return _result(d, warmup_iter)
