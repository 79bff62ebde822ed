"""Annotation markers for kernel signatures (reference: ``core/typing.py:4-10``).

They carry no behaviour: mutation is detected from ``__setitem__`` while
tracing, not from annotations.
"""

from typing import Any

tensor = Any
mutable_tensor = Any
mutable = Any
immutable = Any
