"""Trace + plan + persist: the B200 stand-in for ``compile_to_neff``.

Reference: ``core/compile.py:149-309`` writes the HLO proto, runs
``neuronx-cc`` in a subprocess and returns the NEFF path.  Here the traced
graph goes through ``nkipy_b200.planner.lower`` in process and the plan is
written to ``<build_dir>/<name>_<hash>/<name>.nkbplan`` (plus constants and an
io table).  The hash covers the graph's text form, the planner version and
the collective world size, as the reference's cache key covers the HLO and
the compiler arguments (``runtime/device_kernel.py:38-53``).
"""

import hashlib
import os
import tempfile
import types

import numpy as np

from nkipy_b200.core.trace import NKIPyKernel, _sanitize_array_dtype
from nkipy_b200.planner import lower
from nkipy_b200.spike.runtime import write_plan_files

PLANNER_VERSION = "nkb-planner-2"
PLAN_SUFFIX = ".nkbplan"


def get_build_dir() -> str:
    return os.environ.get("NKB_BUILD_DIR", os.path.join(tempfile.gettempdir(), "nkipy_b200_build"))


def trace(func=None, backend="hlo", **kwargs):
    return NKIPyKernel.trace(func, backend=backend, **kwargs)


def graph_hash(graph, world: int = 1, extra: str = "") -> str:
    h = hashlib.sha256()
    h.update(graph.signature().encode())
    h.update(f"|{PLANNER_VERSION}|world={world}|{extra}".encode())
    return h.hexdigest()[:12]


def specialize(kernel, args, kwargs):
    """Trace ``kernel`` (function or NKIPyKernel) on ndarray arguments."""
    if isinstance(kernel, types.FunctionType):
        kernel = trace(kernel)
    if not isinstance(kernel, NKIPyKernel):
        raise NotImplementedError(f"Unsupported kernel type: {type(kernel)}")
    args = tuple(_sanitize_array_dtype(a, f"arg{i}") if isinstance(a, np.ndarray) else a for i, a in enumerate(args))
    kwargs = {k: _sanitize_array_dtype(v, k) if isinstance(v, np.ndarray) else v for k, v in kwargs.items()}
    kernel.specialize(*args, **kwargs)
    return kernel, kernel._code


def compile_to_plan(kernel, output_dir, name=None, world=1, use_cached_if_exists=True):
    """Plan an already specialised kernel; returns the plan file path."""
    graph = kernel._code
    name = name or kernel.__name__
    path = os.path.join(output_dir, f"{name}{PLAN_SUFFIX}")
    if use_cached_if_exists and os.path.exists(path) and os.path.exists(path + ".io.json"):
        return path
    plan = lower(graph, name=name, world=world)
    write_plan_files(plan, path)
    return path


# reference-compatible name
def compile_to_neff(trace_kernel, output_dir, neff_name=None, world=1, **kwargs):
    name = (neff_name or trace_kernel.__name__).replace(".neff", "")
    return compile_to_plan(trace_kernel, output_dir, name=name, world=world, use_cached_if_exists=False)
