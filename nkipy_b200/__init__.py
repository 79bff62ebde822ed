"""nkipy_b200: NKIPy's NumPy-kernel + tracing API on a B200-native backend.

Kernel bodies stay plain NumPy functions (a direct call runs them on CPU);
``nkipy_b200.core`` traces them, ``nkipy_b200.planner`` lowers the traced graph
onto the sm_100a kernel library of ``libnkb.so``, and ``nkipy_b200.runtime``
(``DeviceKernel``, ``DeviceTensor``, ``baremetal_jit``) runs them.
"""

__version__ = "0.1.0"
