"""Host/device staging shared by the reference-API modules.

A torch CUDA tensor is used where it lives and the results stay on that
device.  Anything else (NumPy arrays, lists, torch CPU tensors) is converted
the way the reference converts it (np.asarray), copied to the current CUDA
device, processed there, and the results are copied back to NumPy.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native as nat


def is_device_tensor(a):
    return isinstance(a, torch.Tensor) and a.is_cuda


def weights_to_device(weights):
    """Returns (w, dtype_code, on_device) with w a contiguous CUDA tensor of
    fp32/fp16/bf16/fp64.  Host inputs of other types are converted to fp32
    first, which is the reference's np.asarray(weights, dtype=np.float32)."""
    if is_device_tensor(weights):
        w = weights
        code = nat.torch_dtype_code(w.dtype)
        if code is None:
            w = w.to(torch.float32)
            code = nat.OQ_F32
        return w.contiguous(), code, True
    if isinstance(weights, torch.Tensor):
        weights = weights.detach().numpy() if weights.dtype != torch.bfloat16 else weights.detach().float().numpy()
    a = np.asarray(weights)
    if nat.numpy_dtype_code(a.dtype) is None:
        a = np.asarray(weights, dtype=np.float32)
    return a, nat.numpy_dtype_code(a.dtype), False


def upload(a, device=None):
    """NumPy array -> contiguous CUDA tensor on `device` (default: current)."""
    nat.require_device()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def to_device(a, device=None):
    if is_device_tensor(a):
        return a.contiguous()
    if isinstance(a, torch.Tensor):
        return a.contiguous().to(device or torch.device("cuda", torch.cuda.current_device()))
    return upload(np.asarray(a), device)


def download(t):
    return t.cpu().numpy()
