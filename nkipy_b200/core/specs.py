"""Kernel specification records (reference: ``core/specs.py:11-92``).

Used by the spec-driven kernel tests: each kernel module lists
``KernelSpec``s whose input shapes/dtypes the tests instantiate.
"""

from dataclasses import dataclass
from typing import Any, List, Optional, Tuple, Type, Union

import numpy as np


@dataclass
class ShapeSpec:
    dims: List[Union[int, Tuple[Optional[int], Optional[int]], None]]
    default: Tuple[int, ...]

    def is_valid(self, shape) -> bool:
        if len(shape) != len(self.dims):
            return False
        for actual, want in zip(shape, self.dims):
            if want is None:
                continue
            if isinstance(want, int) and actual != want:
                return False
            if isinstance(want, tuple):
                lo, hi = want
                if (lo is not None and actual < lo) or (hi is not None and actual > hi):
                    return False
        return True


@dataclass
class TypeSpec:
    allowed: List[Type]
    default: Type

    def is_valid(self, dtype) -> bool:
        return dtype in self.allowed


@dataclass(kw_only=True)
class InputSpec:
    dtype_spec: TypeSpec
    description: str = ""
    default_value: Any = None


@dataclass(kw_only=True)
class ScalarInputSpec(InputSpec):
    description: str = "Scalar input"


@dataclass(kw_only=True)
class TensorInputSpec(InputSpec):
    shape_spec: ShapeSpec
    description: str = "Tensor input"


@dataclass
class KernelSpec:
    function: Any
    inputs: List[InputSpec]
    is_pure_numpy: bool = True
    description: str = ""


class CommonTypes:
    FLOATS = TypeSpec(allowed=[np.float32, np.float16], default=np.float32)
    INTS = TypeSpec(allowed=[np.int8, np.int16, np.int32, np.int64], default=np.int32)
    BOOL = TypeSpec(allowed=[bool], default=bool)
