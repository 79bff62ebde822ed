"""Dtype names used in kernel bodies (reference: ``core/language.py:5-9``).

The reference re-exports NKI's dtype objects; here they are the ``ml_dtypes``
NumPy dtypes, which is what the tracer and the device path carry.
"""

import ml_dtypes
import numpy as np

bfloat16 = np.dtype(ml_dtypes.bfloat16)
float8_e5m2 = np.dtype(ml_dtypes.float8_e5m2)
float8_e4m3 = np.dtype(ml_dtypes.float8_e4m3fn)
