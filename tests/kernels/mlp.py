"""Feed-forward blocks (bf16 weights on the tensor cores, fp32 on CUDA cores)."""

import ml_dtypes
import numpy as np

from nkipy_b200.core.specs import KernelSpec, ShapeSpec, TensorInputSpec, TypeSpec

_BF = TypeSpec(allowed=[np.dtype(ml_dtypes.bfloat16), np.float32], default=np.dtype(ml_dtypes.bfloat16))
_F32 = TypeSpec(allowed=[np.float32], default=np.float32)


def swiglu_mlp(x, w_gate, w_up, w_down):
    g = x @ w_gate
    u = x @ w_up
    return (g * (1.0 / (1.0 + np.exp(-g))) * u) @ w_down


def gelu_mlp(x, w1, b1, w2):
    h = x @ w1 + b1
    return np.tanh(h) @ w2


kernel_specs = [
    KernelSpec(swiglu_mlp, [
        TensorInputSpec(dtype_spec=_BF, shape_spec=ShapeSpec([(1, 512), 256], (128, 256))),
        TensorInputSpec(dtype_spec=_BF, shape_spec=ShapeSpec([256, 512], (256, 512))),
        TensorInputSpec(dtype_spec=_BF, shape_spec=ShapeSpec([256, 512], (256, 512))),
        TensorInputSpec(dtype_spec=_BF, shape_spec=ShapeSpec([512, 256], (512, 256))),
    ], description="SwiGLU MLP, separate gate and up weights"),
    KernelSpec(gelu_mlp, [
        TensorInputSpec(dtype_spec=_F32, shape_spec=ShapeSpec([(1, 128), 64], (24, 64))),
        TensorInputSpec(dtype_spec=_F32, shape_spec=ShapeSpec([64, 96], (64, 96))),
        TensorInputSpec(dtype_spec=_F32, shape_spec=ShapeSpec([96], (96,))),
        TensorInputSpec(dtype_spec=_F32, shape_spec=ShapeSpec([96, 32], (96, 32))),
    ], description="two-layer tanh MLP in fp32"),
]
