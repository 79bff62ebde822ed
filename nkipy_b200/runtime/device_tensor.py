"""``DeviceTensor`` (reference ``runtime/device_tensor.py:48-103``).

A device buffer with NumPy/torch interop: ``from_numpy``, ``from_torch``,
``numpy()``, ``torch()``, ``write_from_numpy``, ``write_from_torch`` (size
mismatch -> ``ValueError``).  ``from_torch`` of a CUDA tensor on this
process's device copies device-to-device instead of staging through host
memory.
"""

import ml_dtypes
import numpy as np

from nkipy_b200.spike import SpikeTensor, _nkb, get_spike_singleton

bfloat16 = np.dtype(ml_dtypes.bfloat16)

try:
    import torch

    torch_to_numpy_type = {
        torch.float16: np.dtype(np.float16),
        torch.float32: np.dtype(np.float32),
        torch.bfloat16: bfloat16,
        torch.int32: np.dtype(np.int32),
        torch.uint32: np.dtype(np.uint32),
        torch.int8: np.dtype(np.int8),
        torch.uint8: np.dtype(np.uint8),
        torch.int16: np.dtype(np.int16),
        torch.bool: np.dtype(np.bool_),
    }
    numpy_to_torch_type = {v: k for k, v in torch_to_numpy_type.items()}
    _TORCH_ENABLED = True
except ImportError:  # pragma: no cover
    _TORCH_ENABLED = False


class DeviceTensor(SpikeTensor):
    @classmethod
    def from_torch(cls, tensor, name: str = None, core_id=None) -> "DeviceTensor":
        if not _TORCH_ENABLED:
            raise ImportError("torch is not available")
        dt = torch_to_numpy_type[tensor.dtype]
        spike = get_spike_singleton()
        if tensor.is_cuda and tensor.device.index == spike.device:
            t = tensor.contiguous()
            n = t.numel() * t.element_size()
            out = cls.empty(tuple(t.shape), dt, name=name, core_id=core_id)
            torch.cuda.current_stream(t.device).synchronize()
            src = spike.wrap_device_memory(t.data_ptr(), n, keepalive=t)
            _nkb.call("nkb_copy", out.tensor_ref.handle, 0, src.handle, 0, n)
            return out
        t = tensor.detach().cpu().contiguous()
        arr = t.view(torch.uint8).numpy() if t.dtype == torch.bfloat16 else t.numpy()
        arr = arr.view(dt).reshape(tuple(t.shape)) if t.dtype == torch.bfloat16 else arr
        out = cls.from_numpy(np.ascontiguousarray(arr), name=name, core_id=core_id)
        return out

    def torch(self):
        if not _TORCH_ENABLED:
            raise ImportError("torch is not available")
        arr = self.numpy()
        if self.dtype == bfloat16:
            return torch.from_numpy(arr.view(np.uint16).astype(np.int16)).view(torch.bfloat16).reshape(self.shape)
        return torch.from_numpy(arr).reshape(self.shape)

    def write_from_torch(self, tensor):
        if not _TORCH_ENABLED:
            raise ImportError("torch is not available")
        t = tensor.detach().cpu().contiguous()
        expected = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        if t.numel() * t.element_size() != expected:
            raise ValueError(f"Size mismatch: source {t.numel() * t.element_size()} bytes, target {expected} bytes")
        raw = t.view(torch.uint8).numpy() if t.dtype == torch.bfloat16 else t.numpy()
        get_spike_singleton().tensor_write_from_pybuffer(self.tensor_ref, np.ascontiguousarray(raw))
