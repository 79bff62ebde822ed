"""One-shot execution of a traced kernel (reference ``runtime/execute.py:23-178``).

``baremetal_run_traced_kernel``: down-cast 64-bit inputs, trace, plan into a
fresh build directory, upload inputs, execute, read outputs back, write
aliased (mutated) parameters back into the caller's arrays, and return the
user-visible outputs (auto-aliased ones dropped): one array, a tuple, or
``None``.
"""

import inspect
import os
import shutil

import numpy as np

from nkipy_b200.core.trace import _sanitize_array_dtype
from nkipy_b200.runtime import compile as C
from nkipy_b200.runtime.device_kernel import DeviceKernel
from nkipy_b200.runtime.device_tensor import DeviceTensor


def _compile_kernel(kernel, *args, artifacts_dir=None, additional_compiler_args="", target=None, **kwargs):
    args = tuple(_sanitize_array_dtype(a, f"arg{i}") if isinstance(a, np.ndarray) else a for i, a in enumerate(args))
    kwargs = {k: _sanitize_array_dtype(v, k) if isinstance(v, np.ndarray) else v for k, v in kwargs.items()}
    kernel.specialize(*args, **kwargs)
    ir = kernel._code
    sig = inspect.signature(kernel.func)
    bound = sig.bind(*args, **kwargs)
    bound.apply_defaults()
    originals = {n: a for n, a in bound.arguments.items() if isinstance(a, np.ndarray)}
    for out in ir.outputs:
        bound.arguments[out.name] = np.empty(out.shape, dtype=out.dtype)
    name = kernel.__name__
    build_dir = artifacts_dir or os.path.join(C.get_build_dir(), name)
    if os.path.exists(build_dir):
        shutil.rmtree(build_dir)
    plan_path = C.compile_to_plan(kernel, build_dir, name=name, world=1, use_cached_if_exists=False)
    return plan_path, name, ir, bound, originals


def _execute_plan(plan_path, name, ir, bound, originals, save_trace=False):
    kernel = DeviceKernel.load_from_neff(plan_path, name)
    alias_by_output = {a.output_index: a for a in ir.aliases}
    ins = {}
    for t in ir.inputs:
        if ".must_alias_input" in t.name:
            arr = originals[t.name.split(".must_alias_input")[0]]
        else:
            arr = bound.arguments[t.name]
        ins[t.name] = DeviceTensor.from_numpy(arr)
    outs = {}
    for i, t in enumerate(ir.outputs):
        if i in alias_by_output:
            outs[t.name] = ins[f"{alias_by_output[i].param_name}.must_alias_input"]
        else:
            outs[t.name] = DeviceTensor.empty(t.shape, t.dtype, name=t.name)
    kernel(inputs=ins, outputs=outs, save_trace=save_trace)
    for i, t in enumerate(ir.outputs):
        res = outs[t.name].numpy()
        if i in alias_by_output:
            a = alias_by_output[i]
            np.copyto(dst=originals[a.param_name], src=res)
            bound.arguments[t.name] = originals[a.param_name]
        else:
            np.copyto(dst=bound.arguments[t.name], src=res)
    auto = ir.auto_aliased_indices
    user = [bound.arguments[o.name] for i, o in enumerate(ir.outputs) if i not in auto]
    if len(user) == 1:
        return user[0]
    if user:
        return tuple(user)
    return None


_execute_neff = _execute_plan


def baremetal_run_traced_kernel(kernel, *args, artifacts_dir=None, save_trace=False, additional_compiler_args="",
                                target=None, **kwargs):
    plan_path, name, ir, bound, originals = _compile_kernel(
        kernel, *args, artifacts_dir=artifacts_dir, additional_compiler_args=additional_compiler_args, target=target,
        **kwargs,
    )
    return _execute_plan(plan_path, name, ir, bound, originals, save_trace=save_trace)
