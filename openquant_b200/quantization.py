"""Per-row symmetric INT8 / packed INT4 quantization on the B200.

Drop-in for openquant/quantization.py (openquant 0.5.0): same dataclass,
same functions, same arguments, errors and output layout.  The arithmetic
runs in the sm_100a kernels of the openquant_b200 library
(oq_quant_int8_rowwise, oq_quant_int4_rowwise, oq_dequant_*); a torch CUDA
tensor input gives torch CUDA tensors back, any other input gives NumPy
arrays back, as the reference does.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import _native as nat
from ._tensors import download, is_device_tensor, to_device, upload, weights_to_device

__all__ = ["QuantizedWeights", "quantize", "dequantize"]


@dataclass
class QuantizedWeights:
    """quantization.py:6-11: data (int8 [N,K] or packed uint8 [ceil(N*K/2)]),
    scales (fp32 [N,1]), bits, shape."""

    data: object
    scales: object
    bits: int
    shape: tuple


def quantize(weights, bits: int = 8):
    """Symmetric per-row quantization (quantization.py:14-59).

    scale[r] = max|w[r]| / qmax (qmax = 127 or 7; 1.0 for a zero row);
    q = clip(rint(w / scale), -qmax, qmax).  INT4 packs the row-major
    flattened matrix two values per byte, low nibble first, padding an odd
    total with a zero nibble.
    """
    if bits not in (4, 8):
        raise ValueError("Only INT4 and INT8 supported")
    w, code, on_device = weights_to_device(weights)
    if w.ndim != 2:
        raise ValueError("Expected a 2D weight matrix")
    rows, cols = (int(s) for s in w.shape)
    shape = tuple(w.shape) if not on_device else (rows, cols)
    if rows > 0 and cols == 0:
        raise ValueError("zero-size array to reduction operation maximum which has no identity")

    if not on_device:
        w = upload(w) if rows * cols else None
    dev = w.device if w is not None else None
    nbytes = rows * cols if bits == 8 else (rows * cols + 1) // 2
    qdtype = torch.int8 if bits == 8 else torch.uint8
    if rows == 0:
        data = torch.empty((0, cols) if bits == 8 else (0,), dtype=qdtype)
        scales = torch.empty((0, 1), dtype=torch.float32)
        if on_device:
            data, scales = data.to(weights.device), scales.to(weights.device)
    else:
        nat.require_device()
        with torch.cuda.device(dev):
            data = torch.empty(nbytes, dtype=qdtype, device=dev)
            scales = torch.empty((rows, 1), dtype=torch.float32, device=dev)
            fn = nat.load().oq_quant_int8_rowwise if bits == 8 else nat.load().oq_quant_int4_rowwise
            nat.check(fn(nat.ptr(w), code, rows, cols, nat.ptr(data), nat.ptr(scales), nat.stream_of(dev)))
        if bits == 8:
            data = data.view(rows, cols)
    if not on_device:
        data, scales = download(data), download(scales)
    return QuantizedWeights(data=data, scales=scales, bits=bits, shape=shape)


def dequantize(result: QuantizedWeights):
    """quantization.py:62-82: q.astype(float32) * scales -> fp32 [N,K]."""
    if result.bits not in (4, 8):
        raise ValueError("Unsupported quantization format")
    rows, cols = (int(s) for s in result.shape)
    on_device = is_device_tensor(result.data)
    if rows * cols == 0:
        out = torch.empty((rows, cols), dtype=torch.float32)
        return out.to(result.data.device) if on_device else out.numpy()
    nat.require_device()
    data = to_device(result.data)
    dev = data.device
    scales = to_device(result.scales, dev).to(torch.float32).reshape(-1)
    if scales.numel() == 1 and rows > 1:
        scales = scales.expand(rows).contiguous()
    if scales.numel() != rows:
        raise ValueError(f"expected {rows} row scales, got {scales.numel()}")
    with torch.cuda.device(dev):
        out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
        if result.bits == 8:
            if data.numel() != rows * cols:
                raise ValueError("INT8 data does not match the shape")
            q = data.view(torch.int8) if data.dtype == torch.uint8 else data.to(torch.int8)
            nat.check(nat.load().oq_dequant_int8_rowwise(nat.ptr(q), nat.ptr(scales), rows, cols,
                                                         nat.ptr(out), nat.stream_of(dev)))
        else:
            packed = data.reshape(-1)
            if packed.dtype != torch.uint8:
                packed = packed.view(torch.uint8) if packed.dtype == torch.int8 else packed.to(torch.uint8)
            if packed.numel() * 2 < rows * cols:
                raise ValueError("INT4 data is shorter than the shape")
            nat.check(nat.load().oq_dequant_int4_rowwise(nat.ptr(packed), nat.ptr(scales), rows, cols,
                                                         nat.ptr(out), nat.stream_of(dev)))
    return out if on_device else download(out)
