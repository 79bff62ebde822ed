"""Kernel bodies with ``kernel_specs`` for the spec-driven device suite
(``tests/test_kernel_specs.py``), in the format of the reference's
``tests/kernels/*.py`` (``nkipy.core.specs.KernelSpec``): plain NumPy
functions that run by direct call on the CPU and trace unchanged."""
