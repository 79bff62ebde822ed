"""``BaremetalExecutor`` / ``CompiledKernel`` (reference ``runtime/baremetal_executor.py:18-202``)."""

import inspect
import os

import numpy as np

from nkipy_b200.runtime.device_kernel import DeviceKernel
from nkipy_b200.runtime.device_tensor import DeviceTensor


class CompiledKernel:
    def __init__(self, traced_kernel, compiled_artifact):
        if not os.path.exists(compiled_artifact):
            raise FileNotFoundError(f"Compiled artifact not found: {compiled_artifact}")
        self.traced_kernel = traced_kernel
        self.compiled_artifact = os.path.abspath(compiled_artifact)
        self.ir = traced_kernel._code


class BaremetalExecutor:
    def __init__(self, verbose: int = 0):
        self.verbose = verbose

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return None

    def _prepare_io_tensors(self, ck: CompiledKernel, dk: DeviceKernel, *args, **kwargs):
        sig = inspect.signature(ck.traced_kernel.func)
        bound = sig.bind(*args, **kwargs)
        bound.apply_defaults()
        originals = {n: a for n, a in bound.arguments.items() if isinstance(a, np.ndarray)}
        inputs = {}
        for t in ck.ir.inputs:
            real = t.name.split(".must_alias_input")[0]
            inputs[t.name] = DeviceTensor.from_numpy(originals.get(real, bound.arguments.get(real)))
        outputs = {t.name: t for t in dk.allocate_output_tensors()}
        for a in ck.ir.aliases:
            outputs[ck.ir.outputs[a.output_index].name] = inputs[f"{a.param_name}.must_alias_input"]
        return inputs, outputs, originals

    def benchmark(self, compiled_kernel, *args, warmup_iterations=5, benchmark_iterations=100, mode="device",
                  artifacts_dir=None, **kwargs):
        dk = DeviceKernel.load_from_neff(compiled_kernel.compiled_artifact, name=compiled_kernel.traced_kernel.__name__)
        ins, outs, _ = self._prepare_io_tensors(compiled_kernel, dk, *args, **kwargs)
        return dk.benchmark(ins, outs, warmup_iter=warmup_iterations, benchmark_iter=benchmark_iterations, mode=mode)

    def run(self, compiled_kernel, *args, save_trace=False, artifacts_dir=None, **kwargs):
        dk = DeviceKernel.load_from_neff(compiled_kernel.compiled_artifact, name=compiled_kernel.traced_kernel.__name__)
        ins, outs, originals = self._prepare_io_tensors(compiled_kernel, dk, *args, **kwargs)
        dk(inputs=ins, outputs=outs, save_trace=save_trace)
        ir = compiled_kernel.ir
        for a in ir.aliases:
            np.copyto(dst=originals[a.param_name], src=outs[ir.outputs[a.output_index].name].numpy())
        auto = ir.auto_aliased_indices
        user = [outs[t.name].numpy() for i, t in enumerate(ir.outputs) if i not in auto]
        if len(user) == 1:
            return user[0]
        return tuple(user) if user else None
