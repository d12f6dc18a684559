"""CPU oracle for the OpenQuant quantize-and-multiply path (test infrastructure).

This module is the checker, not the product: only tests, the smoke check and
the CPU-baseline leg of bench.py import it.  It restates, in NumPy, the
algorithms of the reference package (openquant 0.5.0) line by line, so that
the CUDA kernels can be compared with it on the same seeded inputs:

  quantize / dequantize            openquant/quantization.py:14-82
  quantize_int4_groupwise          openquant/groupwise.py:13-61
  dequantize_int4_groupwise        openquant/groupwise.py:64-89
  decode_gpu                       openquant/gpu_benchmark.py:10-30
  restore_groupwise_torch          openquant/group_benchmark.py:11-30
  int4_linear (its arithmetic)     openquant/triton_int4.py:6-75

Parity is pinned: tests/test_oracle.py checks every function here against the
golden vectors in tests/golden/, which tests/golden/make_golden.py produced by
running the reference package itself.

All arithmetic follows the reference: fp32 IEEE division for the scales and
quotients, np.rint (round half to even), clipping to +-qmax, and the nibble
layout (element 2i in the low nibble of byte i).
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

__all__ = [
    "quantize",
    "dequantize",
    "quantize_int4_groupwise",
    "dequantize_int4_groupwise",
    "round_to_dtype",
    "int4_linear",
    "padded_cols",
    "threaded_rows",
]


def quantize(weights, bits=8):
    """Per-row symmetric quantizer; returns (data, scales).

    quantization.py:15-21 validation, :23 qmax, :25-31 per-row scale
    max|w|/qmax in fp32 (1.0 for a zero row), :33-37 clip(rint(w/s)) to int8,
    :39-52 INT4 packing of the flattened matrix (odd totals padded with 0).
    """
    if bits not in (4, 8):
        raise ValueError("Only INT4 and INT8 supported")
    w = np.asarray(weights, dtype=np.float32)
    if w.ndim != 2:
        raise ValueError("Expected a 2D weight matrix")
    qmax = (1 << (bits - 1)) - 1
    with np.errstate(all="ignore"):
        peak = np.max(np.abs(w), axis=1, keepdims=True)
        scales = np.where(peak == 0, np.float32(1.0), peak / np.float32(qmax)).astype(np.float32)
        quot = np.rint(w / scales)
        quot = np.clip(quot, -qmax, qmax)
        # NaN quotients (0/0, inf/inf, NaN inputs) become 0, which is what
        # the reference's astype(np.int8) produces for them on x86-64.
        quot = np.where(np.isnan(quot), np.float32(0), quot)
    q = quot.astype(np.int8)
    if bits == 8:
        return q, scales
    flat = q.reshape(-1)
    if flat.size % 2:
        flat = np.concatenate([flat, np.zeros(1, np.int8)])
    nib = flat.astype(np.uint8) & 0x0F
    data = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)
    return data, scales


def _unpack_signed(packed):
    """Two's-complement nibbles -> int16, element 2i from the low nibble."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(p.size * 2, dtype=np.int16)
    out[0::2] = p & 0x0F
    out[1::2] = p >> 4
    return np.where(out >= 8, out - 16, out)


def dequantize(data, scales, bits, shape):
    """quantization.py:62-82: q.astype(f32) * scales (row scales broadcast)."""
    rows, cols = shape
    if bits == 8:
        q = np.asarray(data).reshape(shape)
    elif bits == 4:
        q = _unpack_signed(data)[: rows * cols].reshape(shape)
    else:
        raise ValueError("Unsupported quantization format")
    return q.astype(np.float32) * np.asarray(scales, dtype=np.float32).reshape(rows, -1)


def padded_cols(cols, group_size):
    """groupwise.py:27-29: K rounded up to a multiple of the group."""
    return ((cols + group_size - 1) // group_size) * group_size


def quantize_int4_groupwise(weights, group_size=32):
    """groupwise.py:13-61; returns (data, scales)."""
    a = np.asarray(weights, dtype=np.float32)
    if a.ndim != 2 or min(a.shape) == 0:
        raise ValueError("Expected nonempty 2D weights")
    if group_size < 2 or group_size % 2 != 0:
        raise ValueError("Group size must be even and >= 2")
    if not np.isfinite(a).all():
        raise ValueError("Weights must be finite")
    rows, cols = a.shape
    kp = padded_cols(cols, group_size)
    padded = np.zeros((rows, kp), dtype=np.float32)
    padded[:, :cols] = a
    blocks = padded.reshape(rows, kp // group_size, group_size)
    scales = np.max(np.abs(blocks), axis=2) / np.float32(7.0)
    scales = np.where(scales == 0, np.float32(1.0), scales).astype(np.float32)
    q = np.clip(np.rint(blocks / scales[:, :, None]), -7, 7).astype(np.int8).reshape(-1)
    nib = q.astype(np.uint8) & 15
    data = (nib[0::2] | (nib[1::2] << 4)).astype(np.uint8)
    return data, scales


def dequantize_int4_groupwise(data, scales, shape, group_size):
    """groupwise.py:64-89: signed nibble * group scale, cropped to K."""
    rows, cols = shape
    signed = _unpack_signed(data).astype(np.float32)
    blocks = signed.reshape(rows, -1, group_size)
    restored = (blocks * np.asarray(scales, dtype=np.float32)[:, :, None]).reshape(rows, -1)
    return restored[:, :cols]


def round_to_dtype(a, dtype):
    """Round fp32 values to fp16 or bf16 (round to nearest, ties to even)
    and return them widened back to fp32.  This is the `.to(tl.float16)` of
    triton_int4.py:63-65 and the `.half()` of tests/test_triton_int4.py:45-51;
    bf16 uses the same rounding on the top 16 bits of the fp32 pattern."""
    a = np.asarray(a, dtype=np.float32)
    if dtype in ("f16", "float16", np.float16):
        # beyond the fp16 range the value becomes +-inf, as torch's .half() does
        with np.errstate(over="ignore"):
            return a.astype(np.float16).astype(np.float32)
    if dtype in ("bf16", "bfloat16"):
        u = a.view(np.uint32).astype(np.uint64)
        lsb = (u >> 16) & 1
        r = ((u + 0x7FFF + lsb) >> 16) << 16
        r = r.astype(np.uint32)
        nan = np.isnan(a)
        r[nan] = (a.view(np.uint32)[nan] | 0x00400000) & 0xFFFF0000
        return r.view(np.float32)
    if dtype in ("f32", "float32", np.float32):
        return a
    raise ValueError(f"unknown dtype {dtype!r}")


def int4_linear(x, data, scales, out_features, group_size, x_dtype="f16"):
    """The arithmetic of triton_int4.py:6-75 on the CPU.

    W[n,k] = round_to_x_dtype(int4(n,k) * scale[n, k//g]) computed in fp32
    (triton_int4.py:62-65); y = x . W^T.  The products of two fp16/bf16
    values are exact in fp64 and the fp64 sum is accurate to ~1e-16, so this
    is the exactly-rounded result the fp32-accumulating kernels approximate.
    """
    x = round_to_dtype(np.asarray(x, dtype=np.float32), x_dtype)
    k = x.shape[1]
    w = dequantize_int4_groupwise(data, scales, (out_features, k), group_size)
    w = round_to_dtype(w, x_dtype)
    return (x.astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


def threaded_rows(fn, rows, threads=None, min_rows=64):
    """Run fn(r0, r1) over row blocks on a thread pool and return the list of
    results.  NumPy releases the GIL inside ufuncs, so the row-independent
    steps of the oracle scale over host cores this way."""
    threads = threads or len(os.sched_getaffinity(0))
    blocks = max(1, min(threads, rows // max(1, min_rows)))
    edges = np.linspace(0, rows, blocks + 1).astype(int)
    if blocks == 1:
        return [fn(0, rows)]
    with ThreadPoolExecutor(max_workers=blocks) as pool:
        return list(pool.map(lambda i: fn(edges[i], edges[i + 1]), range(blocks)))


def int8_matmul(qx, sx, qw, sw):
    """y[m, n] = sx[m] * sw[n] * sum_k qx[m, k] qw[n, k] in float64.

    The W8A8 product of two per-row INT8 operands in the format of quantize
    (quantization.py:23-37).  The integer sums are exact in float64 while
    K * 127^2 < 2^53.
    """
    qx = np.asarray(qx, dtype=np.float64)
    qw = np.asarray(qw, dtype=np.float64)
    sx = np.asarray(sx, dtype=np.float64).reshape(-1, 1)
    sw = np.asarray(sw, dtype=np.float64).reshape(1, -1)
    return (qx @ qw.T) * sx * sw
