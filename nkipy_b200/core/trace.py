"""``NKIPyKernel``: trace a NumPy kernel body into a ``TraceGraph``.

Same contract as the reference's ``nkipy/core/trace.py:50-250``:

* ``NKIPyKernel.trace(func, backend="hlo")`` wraps a plain function (also
  usable as a decorator); the function stays callable on ndarrays directly;
* ``specialize(*args, **kwargs)`` binds the arguments, turns every ndarray
  argument into a graph parameter named after the Python parameter (float64 /
  int64 / uint64 arrays are down-cast with a warning), runs the body, and
  records outputs;
* outputs are named ``output{i}``; a parameter mutated through ``__setitem__``
  is renamed ``<name>.must_alias_input``, its final value becomes an output
  named ``<name>`` (appended when the body did not return it), and an
  ``AliasInfo`` records the pair; a returned, unmutated parameter gets an
  explicit ``copy``.
"""

import inspect
import warnings

import numpy as np

from nkipy_b200.core.backend import tracing
from nkipy_b200.core.dispatch import register_all_numpy_apis
from nkipy_b200.core.graph import AliasInfo, TraceContext, TraceGraph, get_trace_context
from nkipy_b200.core.tensor import NKIPyTensorRef

register_all_numpy_apis()

_DOWNCAST = {
    np.dtype("float64"): np.dtype("float32"),
    np.dtype("int64"): np.dtype("int32"),
    np.dtype("uint64"): np.dtype("uint32"),
}


def _sanitize_array_dtype(arr: np.ndarray, name: str = "") -> np.ndarray:
    target = _DOWNCAST.get(arr.dtype)
    if target is None:
        return arr
    label = f" '{name}'" if name else ""
    warnings.warn(
        f"Input tensor{label} has dtype {arr.dtype} which the device path does not carry. "
        f"Automatically casting to {target}.",
        stacklevel=3,
    )
    return arr.astype(target)


class NKIPyKernel:
    def __init__(self, func, backend="hlo", **kwargs):
        self.func = func
        self.backend = backend
        self._code = None

    @property
    def __name__(self):
        return self.func.__name__

    def __repr__(self):
        return f"<NKIPyKernel '{self.func.__name__}' backend='{self.backend}'>"

    def __call__(self, *args, **kwargs):
        # A traced kernel is still a NumPy function: calling it runs on CPU.
        return self.func(*args, **kwargs)

    def specialize(self, *args, **kwargs):
        if self.backend == "hlo":
            return self._specialize(*args, **kwargs)
        if self.backend == "cpu":
            print("CPU backend does not require specialization")
            return None
        raise ValueError(f"Unknown backend {self.backend}")

    @staticmethod
    def _param(shape, dtype, name):
        ctx = get_trace_context()
        return NKIPyTensorRef(ctx.module.add_parameter(shape, dtype, name=name), name=name)

    def _specialize(self, *args, **kwargs):
        graph = TraceGraph(name=self.func.__name__)
        with tracing(TraceContext(graph)):
            sig = inspect.signature(self.func)
            bound = sig.bind(*args, **kwargs)
            bound.apply_defaults()
            call_args, call_kwargs, params = [], {}, []
            for name, arg in bound.arguments.items():
                kind = sig.parameters[name].kind
                if isinstance(arg, np.ndarray):
                    arg = _sanitize_array_dtype(arg, name)
                    ref = self._param(arg.shape, arg.dtype, name)
                    ref._original_parameter = ref.backend_tensor
                    params.append((name, ref))
                    value = ref
                else:
                    value = arg
                if kind in (inspect.Parameter.POSITIONAL_ONLY, inspect.Parameter.POSITIONAL_OR_KEYWORD):
                    call_args.append(value)
                elif kind == inspect.Parameter.KEYWORD_ONLY:
                    call_kwargs[name] = value
                elif kind == inspect.Parameter.VAR_POSITIONAL:
                    for item in arg if isinstance(arg, (list, tuple)) else [arg]:
                        if isinstance(item, np.ndarray):
                            item = _sanitize_array_dtype(item, f"{name}_item")
                            call_args.append(self._param(item.shape, item.dtype, f"{name}_item"))
                        else:
                            call_args.append(item)
                elif kind == inspect.Parameter.VAR_KEYWORD:
                    for k, v in (arg or {}).items():
                        if isinstance(v, np.ndarray):
                            v = _sanitize_array_dtype(v, k)
                            call_kwargs[k] = self._param(v.shape, v.dtype, k)
                        else:
                            call_kwargs[k] = v
            ret = self.func(*call_args, **call_kwargs)
            self._mark_outputs(graph, ret, params)
            self._code = graph
        return graph

    @staticmethod
    def _mark_outputs(graph: TraceGraph, ret, params):
        if ret is None:
            ret = []
        elif not isinstance(ret, (list, tuple)):
            ret = [ret]
        ret = list(ret)
        n_user = len(ret)
        ctx = get_trace_context()

        aliased = {}
        for name, ref in params:
            if not ref._is_mutated:
                continue
            pidx = None
            for p in graph.parameters:
                if p.name == name:
                    p.name = f"{name}.must_alias_input"
                    pidx = p.parameter_id
                    break
            if pidx is None:
                raise RuntimeError(f"Mutated parameter '{name}' not found in graph parameters")
            pos = next((i for i, r in enumerate(ret) if r is ref), None)
            if pos is None:
                ret.append(ref)
                pos = len(ret) - 1
            aliased[pos] = (name, pidx)

        for i, r in enumerate(ret):
            if isinstance(r, NKIPyTensorRef) and i not in aliased and r.backend_tensor.is_parameter:
                bt = r.backend_tensor
                ret[i] = NKIPyTensorRef(ctx.build_op("copy", [bt], bt.shape, bt.dtype), name="")

        for i, r in enumerate(ret):
            if not isinstance(r, NKIPyTensorRef):
                raise RuntimeError(f"Unexpected return value type: {type(r)}")
            if i in aliased:
                pname, pidx = aliased[i]
                graph.aliases.append(
                    AliasInfo(output_index=i, param_index=pidx, param_name=pname, is_user_returned=i < n_user)
                )
                r.backend_tensor.name = pname
            if not r.backend_tensor.name:
                r.backend_tensor.name = f"output{i}"
        graph.set_results([r.backend_tensor for r in ret])

    @classmethod
    def trace(cls, func=None, backend="hlo", **kwargs):
        if func is None:
            return lambda f: cls(f, backend, **kwargs)
        return cls(func, backend, **kwargs)


trace = NKIPyKernel.trace
