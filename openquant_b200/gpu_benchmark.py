"""decode_gpu: per-row INT8 / INT4 decode on the B200.

Drop-in for openquant/gpu_benchmark.py:10-30.  The reference decodes with
about six eager torch kernels; here one sm_100a kernel
(oq_dequant_int8_rowwise / oq_dequant_int4_rowwise) writes the fp32 result.
CUDA tensors are decoded where they live; CPU tensors are copied to the
current GPU, decoded there and the result is copied back (a CPU tensor in,
a CPU tensor out, as the reference's tests expect).
"""
from __future__ import annotations

import torch

from . import _native as nat

__all__ = ["decode_gpu"]


def decode_gpu(data, scales, bits, shape):
    """Returns fp32 values * scales with the given (rows, cols) shape."""
    if bits not in (4, 8):
        raise ValueError("Expected 4 or 8 bits")
    rows, cols = (int(s) for s in shape)
    home = data.device if isinstance(data, torch.Tensor) else torch.device("cpu")
    nat.require_device()
    dev = home if home.type == "cuda" else torch.device("cuda", torch.cuda.current_device())
    d = torch.as_tensor(data).to(dev).contiguous().reshape(-1)
    s = torch.as_tensor(scales).to(dev).to(torch.float32).contiguous().reshape(-1)
    if s.numel() == 1 and rows > 1:
        s = s.expand(rows).contiguous()
    if s.numel() != rows:
        raise ValueError(f"expected {rows} row scales, got {s.numel()}")
    with torch.cuda.device(dev):
        out = torch.empty((rows, cols), dtype=torch.float32, device=dev)
        if rows * cols:
            if bits == 8:
                if d.numel() != rows * cols:
                    raise ValueError("INT8 data does not match the shape")
                q = d.view(torch.int8) if d.dtype == torch.uint8 else d.to(torch.int8)
                nat.check(nat.load().oq_dequant_int8_rowwise(nat.ptr(q), nat.ptr(s), rows, cols, nat.ptr(out),
                                                             nat.stream_of(dev)))
            else:
                p = d if d.dtype == torch.uint8 else d.to(torch.uint8)
                if p.numel() * 2 < rows * cols:
                    raise ValueError("INT4 data is shorter than the shape")
                nat.check(nat.load().oq_dequant_int4_rowwise(nat.ptr(p), nat.ptr(s), rows, cols, nat.ptr(out),
                                                             nat.stream_of(dev)))
    return out if home.type == "cuda" else out.cpu()
