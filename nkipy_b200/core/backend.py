"""Active-trace bookkeeping.

Mirrors the reference's ``nkipy/core/backend/__init__.py:21-58``: a single
process-wide trace context, ``tracing(ctx)`` to activate it, and
``get_backend()`` which answers ``"cpu"`` when no trace is active (so ops
called outside a trace run their NumPy implementation) or the context's
``backend_name`` while tracing.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Optional, Tuple

_active_ctx = None


@contextmanager
def tracing(ctx):
    """Make ``ctx`` the active trace context for the duration of the block."""
    global _active_ctx
    previous = _active_ctx
    _active_ctx = ctx
    try:
        yield ctx
    finally:
        _active_ctx = previous


def active_context():
    return _active_ctx


def get_backend() -> str:
    """``"cpu"`` outside a trace, otherwise the active context's backend name."""
    if _active_ctx is None:
        return "cpu"
    return _active_ctx.backend_name


def set_source_location(location: Optional[Tuple[str, int]]) -> None:
    """Record the user source line that the next graph node comes from."""
    if _active_ctx is not None:
        _active_ctx.set_source_location(location)
