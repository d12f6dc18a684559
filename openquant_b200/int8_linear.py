"""W8A8 linear layer: per-token INT8 activations times per-row INT8 weights on
the B200's tcgen05 tensor cores (int32 sums).

The weights are the reference's per-row INT8 format (quantize(w, bits=8),
openquant/quantization.py:14-40: int8 data, one fp32 scale max|w|/127 per
row).  The activations get the same quantization per token (row of x), done
on the GPU by the same kernel, so

    y[m, n] = sx[m] * sw[n] * sum_k qx[m, k] * qw[n, k]

with the integer products summed exactly.  The reference stops at weight-only
quantization; this is the activation-side extension of its INT8 format.
"""
from __future__ import annotations

import torch

from . import _native as nat
from .quantization import QuantizedWeights

__all__ = ["quantize_activations", "int8_matmul", "int8_linear"]

_CODES = {torch.float32: nat.OQ_F32, torch.float16: nat.OQ_F16, torch.bfloat16: nat.OQ_BF16}


def quantize_activations(x):
    """Per-token INT8: (qx int8 [M, K], sx fp32 [M]) for a CUDA x [M, K]
    (fp32, fp16 or bf16), bit for bit the reference's quantize(x, 8) with one
    row per token."""
    if not isinstance(x, torch.Tensor) or not x.is_cuda or x.ndim != 2:
        raise ValueError("x must be a 2D CUDA tensor")
    if x.dtype not in _CODES:
        raise ValueError("x must be fp32, fp16 or bf16")
    m, k = (int(v) for v in x.shape)
    if m < 1 or k < 1:
        raise ValueError("Matrix dimensions must be positive")
    x = x.contiguous()
    nat.require_device()
    with torch.cuda.device(x.device):
        qx = torch.empty((m, k), dtype=torch.int8, device=x.device)
        sx = torch.empty((m,), dtype=torch.float32, device=x.device)
        nat.check(nat.load().oq_quant_int8_rowwise(nat.ptr(x), _CODES[x.dtype], m, k, nat.ptr(qx), nat.ptr(sx),
                                                   nat.stream_of(x.device)))
    return qx, sx


def int8_matmul(qx, sx, qw, sw, *, out=None):
    """y = (qx . qw^T) * sx[:, None] * sw[None, :] in fp32 on the tensor cores.

    qx int8 [M, K], sx fp32 [M] (or [M, 1]), qw int8 [N, K], sw fp32 [N] (or
    [N, 1]), all on one GPU; K % 16 == 0.  Asynchronous on the current stream.
    """
    for t in (qx, sx, qw, sw):
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise ValueError("All tensors must be on CUDA")
    if qx.dtype != torch.int8 or qw.dtype != torch.int8:
        raise ValueError("qx and qw must be int8")
    if sx.dtype != torch.float32 or sw.dtype != torch.float32:
        raise ValueError("Scales must be float32")
    if qx.ndim != 2 or qw.ndim != 2 or qx.shape[1] != qw.shape[1]:
        raise ValueError("qx [M, K] and qw [N, K] must share K")
    m, k = (int(v) for v in qx.shape)
    n = int(qw.shape[0])
    if sx.numel() != m or sw.numel() != n:
        raise ValueError("Incorrect scales shape")
    if k % 16:
        raise ValueError("K must be a multiple of 16")
    if len({t.device for t in (qx, sx, qw, sw)}) != 1:
        raise ValueError("All tensors must use the same GPU")
    qx, qw, sx, sw = qx.contiguous(), qw.contiguous(), sx.contiguous(), sw.contiguous()
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=qx.device)
    elif out.shape != (m, n) or out.dtype != torch.float32 or out.device != qx.device or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 (M, N) tensor on the operands' GPU")
    nat.require_device()
    with torch.cuda.device(qx.device):
        nat.check(nat.load().oq_int8_gemm(nat.ptr(qx), nat.ptr(sx), nat.ptr(qw), nat.ptr(sw), nat.ptr(out), m, n, k,
                                          nat.stream_of(qx.device)))
    return out


def int8_linear(x, weights: QuantizedWeights, *, out=None):
    """y = x . W^T with x quantized per token to INT8 and W given as
    quantize(w, bits=8) on the same GPU (data int8 [N, K], scales [N, 1])."""
    if weights.bits != 8:
        raise ValueError("int8_linear needs INT8 per-row weights (quantize(w, bits=8))")
    qx, sx = quantize_activations(x)
    return int8_matmul(qx, sx, weights.data, weights.scales.reshape(-1), out=out)
