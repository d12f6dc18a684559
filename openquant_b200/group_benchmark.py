"""restore_groupwise_torch: groupwise INT4 -> fp32 on the B200.

Drop-in for openquant/group_benchmark.py:11-30 (one sm_100a kernel,
oq_dequant_int4_group, instead of the reference's eager torch ops).  CUDA
tensors are restored where they live; CPU tensors are copied to the current
GPU and the result is copied back.
"""
from __future__ import annotations

import torch

from . import _native as nat
from .groupwise import padded_cols

__all__ = ["restore_groupwise_torch"]


def restore_groupwise_torch(data, scales, shape, group_size):
    """fp32 (rows, cols): signed nibble * scales[row, col // group_size]."""
    rows, cols = (int(s) for s in shape)
    g = int(group_size)
    if g < 2 or g % 2:
        raise ValueError("Group size must be even and >= 2")
    home = data.device if isinstance(data, torch.Tensor) else torch.device("cpu")
    nat.require_device()
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    d = torch.as_tensor(data).to(dev).contiguous().reshape(-1)
    s = torch.as_tensor(scales).to(dev).to(torch.float32).contiguous()
    kp = padded_cols(cols, g)
    if d.dtype != torch.uint8 or d.numel() != rows * kp // 2:
        raise ValueError("Incorrect packed weight count")
    if s.numel() != rows * (kp // g):
        raise ValueError("Incorrect scales shape")
    with torch.cuda.device(dev):
        out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
        nat.check(nat.load().oq_dequant_int4_group(nat.ptr(d), nat.ptr(s), rows, cols, g, nat.ptr(out),
                                                   nat.stream_of(dev)))
    return out if home.type == "cuda" else out.cpu()
