"""Backward-compatible entry points (reference: ``core/tensor_apis.py``)."""

from nkipy_b200.core.ops import constant, conv2d, conv3d, full, rms_norm, softmax, topk, zeros

__all__ = ["constant", "conv2d", "conv3d", "topk", "rms_norm", "softmax", "zeros", "full"]
