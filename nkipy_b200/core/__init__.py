"""Tracing frontend: NumPy kernel body -> ``TraceGraph``."""

from nkipy_b200.core.trace import NKIPyKernel, trace  # noqa: F401
