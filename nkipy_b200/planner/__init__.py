"""Fusion/tiling pass: traced graph -> libnkb launch plan."""

from nkipy_b200.planner.lower import lower  # noqa: F401
from nkipy_b200.planner.plan import Plan  # noqa: F401
