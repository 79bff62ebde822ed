"""Runtime API (reference ``nkipy/runtime/__init__.py``): same public names."""

from nkipy_b200.runtime.baremetal_executor import BaremetalExecutor, CompiledKernel
from nkipy_b200.runtime.decorators import baremetal_jit
from nkipy_b200.runtime.device_kernel import DeviceKernel
from nkipy_b200.runtime.device_tensor import DeviceTensor
from nkipy_b200.runtime.execute import baremetal_run_traced_kernel
from nkipy_b200.runtime.utils import is_b200_compatible, is_neuron_compatible

__all__ = [
    "BaremetalExecutor",
    "CompiledKernel",
    "DeviceKernel",
    "DeviceTensor",
    "baremetal_jit",
    "baremetal_run_traced_kernel",
    "is_b200_compatible",
    "is_neuron_compatible",
]
