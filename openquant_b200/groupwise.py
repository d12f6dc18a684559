"""Groupwise INT4 quantization on the B200.

Drop-in for openquant/groupwise.py (openquant 0.5.0).  The arithmetic runs
in oq_quant_int4_group / oq_dequant_int4_group (sm_100a).  A torch CUDA
tensor input gives torch CUDA tensors back; any other input gives NumPy
arrays back, as the reference does.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import _native as nat
from ._tensors import download, is_device_tensor, to_device, upload, weights_to_device

__all__ = ["Groupwise4", "quantize_int4_groupwise", "dequantize_int4_groupwise", "padded_cols"]


@dataclass(frozen=True)
class Groupwise4:
    """groupwise.py:5-10: data (uint8 [N*KP/2]), scales (fp32 [N, KP/g]),
    shape (N, K), group_size."""

    data: object
    scales: object
    shape: tuple
    group_size: int


def padded_cols(cols, group_size):
    """KP: K rounded up to a multiple of the group (groupwise.py:27-29)."""
    return ((cols + group_size - 1) // group_size) * group_size


def quantize_int4_groupwise(weights, group_size=32):
    """groupwise.py:13-61.

    Rows are zero-padded to KP; each group of `group_size` columns gets
    scale = max|w| / 7 (1.0 for an all-zero group) and
    q = clip(rint(w / scale), -7, 7), packed two per byte, low nibble first.
    Raises ValueError for non-2-D or empty input, an odd or < 2 group size,
    and non-finite weights, in that order.
    """
    w, code, on_device = weights_to_device(weights)
    if w.ndim != 2 or min(w.shape) == 0:
        raise ValueError("Expected nonempty 2D weights")
    if group_size < 2 or group_size % 2 != 0:
        raise ValueError("Group size must be even and >= 2")
    group_size = int(group_size)
    rows, cols = (int(s) for s in w.shape)
    kp = padded_cols(cols, group_size)
    if not on_device:
        w = upload(w)
    nat.require_device()
    dev = w.device
    with torch.cuda.device(dev):
        data = torch.empty(rows * kp // 2, dtype=torch.uint8, device=dev)
        scales = torch.empty((rows, kp // group_size), dtype=torch.float32, device=dev)
        flag = torch.empty(1, dtype=torch.int32, device=dev)
        nat.check(nat.load().oq_quant_int4_group(nat.ptr(w), code, rows, cols, group_size, nat.ptr(data),
                                                 nat.ptr(scales), nat.ptr(flag), nat.stream_of(dev)))
        if int(flag.item()) != 0:
            raise ValueError("Weights must be finite")
    if not on_device:
        data, scales = download(data), download(scales)
    return Groupwise4(data=data, scales=scales, shape=(rows, cols), group_size=group_size)


def dequantize_int4_groupwise(q):
    """groupwise.py:64-89: signed nibble * group scale, fp32 [N, K]."""
    rows, cols = (int(s) for s in q.shape)
    g = int(q.group_size)
    on_device = is_device_tensor(q.data)
    nat.require_device()
    data = to_device(q.data).reshape(-1)
    dev = data.device
    scales = to_device(q.scales, dev)
    kp = padded_cols(cols, g)
    if data.dtype != torch.uint8:
        raise ValueError("packed data must be uint8")
    if data.numel() != rows * kp // 2:
        raise ValueError("Incorrect packed weight count")
    if scales.dtype != torch.float32 or scales.numel() != rows * (kp // g):
        raise ValueError("Incorrect scales shape")
    scales = scales.contiguous()
    with torch.cuda.device(dev):
        out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
        nat.check(nat.load().oq_dequant_int4_group(nat.ptr(data), nat.ptr(scales), rows, cols, g,
                                                   nat.ptr(out), nat.stream_of(dev)))
    return out if on_device else download(out)
