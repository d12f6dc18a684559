"""`openquant report`: reproducible quantization report.

make_cpu_report: JSON schema 1, the same fields as openquant/report.py:13-90
(FP32 / INT8 / INT4 / INT4_GROUP_g storage, compression, error), computed
through the B200 kernels; "device" names the GPU that computed it.

make_gpu_report (`openquant report --gpu`): JSON schema 2 = schema 1 plus,
per format, the device time and bandwidth of its quantize and dequantize
kernels and of the fused product with a batch of activations (INT4_GROUP:
the INT4 dequant-GEMV / GEMM; INT8: the W8A8 tensor-core GEMM), each the
median of 40 CUDA-event-timed calls after 10 warm-ups (the reference
benchmark's statistic, openquant/fused_benchmark.py:14-34).
"""
import platform
from datetime import datetime, timezone

import numpy as np

from .groupwise import dequantize_int4_groupwise, quantize_int4_groupwise
from .quantization import dequantize, quantize

__all__ = ["make_cpu_report", "make_gpu_report"]


def make_cpu_report(rows=1024, cols=1024, seed=42, group_size=32):
    if rows < 1 or cols < 1:
        raise ValueError("Dimensions must be positive")
    if group_size < 2 or group_size % 2:
        raise ValueError("Group size must be even and >= 2")
    import torch

    rng = np.random.default_rng(seed)
    weights = rng.normal(0, 0.2, (rows, cols)).astype(np.float32)
    baseline_bytes = weights.nbytes
    formats = {}

    def add_result(name, restored, stored_bytes):
        error = np.linalg.norm(weights - restored) / np.linalg.norm(weights)
        formats[name] = {
            "storage_bytes": int(stored_bytes),
            "compression_ratio": round(baseline_bytes / stored_bytes, 4),
            "memory_reduction_pct": round(100 * (1 - stored_bytes / baseline_bytes), 4),
            "relative_weight_error_pct": round(100 * float(error), 6),
        }

    add_result("FP32", weights, baseline_bytes)
    for bits in (8, 4):
        q = quantize(weights, bits)
        add_result(f"INT{bits}", dequantize(q), q.data.nbytes + q.scales.nbytes)
    q = quantize_int4_groupwise(weights, group_size)
    add_result(f"INT4_GROUP_{group_size}", dequantize_int4_groupwise(q), q.data.nbytes + q.scales.nbytes)
    return {
        "schema_version": 1,
        "project": "OpenQuant",
        "version": "0.5.0",
        "generated_at_utc": datetime.now(timezone.utc).isoformat(),
        "device": f"cuda ({torch.cuda.get_device_name()})",
        "python": platform.python_version(),
        "numpy": np.__version__,
        "seed": seed,
        "weights": {"shape": [rows, cols], "dtype": "float32", "distribution": "normal(0, 0.2)"},
        "formats": formats,
    }


def _median_us(fn, warmup=10, iters=40):
    import torch

    for _ in range(warmup):
        fn()
    times = []
    for _ in range(iters):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        fn()
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end) * 1e3)
    return float(np.median(times))


def make_gpu_report(rows=4096, cols=4096, seed=42, group_size=128, batch=1):
    """Schema-2 report: make_cpu_report's formats and errors for a
    `rows` x `cols` matrix, plus GPU timings of each format's kernels on
    that matrix (weights and activations resident on the GPU)."""
    if batch < 1:
        raise ValueError("Batch must be positive")
    import torch

    from . import _native as nat
    from .int8_linear import int8_linear
    from .triton_int4 import int4_linear

    base = make_cpu_report(rows=rows, cols=cols, seed=seed, group_size=group_size)
    nat.require_device()
    dev = torch.device("cuda", torch.cuda.current_device())
    rng = np.random.default_rng(seed)
    w = torch.from_numpy(rng.normal(0, 0.2, (rows, cols)).astype(np.float32)).to(dev)
    x = torch.from_numpy(rng.normal(0, 1.0, (batch, cols)).astype(np.float32)).to(dev)
    w16, x16 = w.half(), x.half()

    def entry(us, nbytes, flops=None):
        out = {"time_us": round(us, 3), "bytes": int(nbytes), "GB_per_s": round(nbytes / us / 1e3, 2)}
        if flops is not None:
            out["TFLOP_per_s"] = round(flops / us / 1e6, 3)
        return out

    gpu = {}
    n_el = rows * cols
    for bits in (8, 4):
        q = quantize(w16, bits)
        qbytes = q.data.numel() * q.data.element_size() + q.scales.numel() * 4
        gpu[f"INT{bits}"] = {
            "quantize_fp16": entry(_median_us(lambda: quantize(w16, bits)), n_el * 2 + qbytes),
            "dequantize": entry(_median_us(lambda: dequantize(q)), qbytes + n_el * 4),
        }
        if bits == 8 and cols % 16 == 0:
            gpu["INT8"]["w8a8_linear"] = entry(_median_us(lambda: int8_linear(x16, q)),
                                               qbytes + batch * cols * 2 + batch * rows * 4, 2.0 * batch * rows * cols)
    qg = quantize_int4_groupwise(w16, group_size)
    gbytes = qg.data.numel() + qg.scales.numel() * 4
    gpu[f"INT4_GROUP_{group_size}"] = {
        "quantize_fp16": entry(_median_us(lambda: quantize_int4_groupwise(w16, group_size)), n_el * 2 + gbytes),
        "dequantize": entry(_median_us(lambda: dequantize_int4_groupwise(qg)), gbytes + n_el * 4),
        "int4_linear": entry(_median_us(lambda: int4_linear(x16, qg.data, qg.scales, rows, group_size)),
                             gbytes + batch * cols * 2 + batch * rows * 4, 2.0 * batch * rows * cols),
    }
    props = torch.cuda.get_device_properties(dev)
    base.update({
        "schema_version": 2,
        "gpu": {
            "name": props.name,
            "sm_count": props.multi_processor_count,
            "memory_gb": round(props.total_memory / 1e9, 1),
            "library": nat.load().oq_version().decode(),
            "batch": batch,
            "timing": "median of 40 CUDA-event-timed calls after 10 warm-ups, inputs on the GPU",
            "formats": gpu,
        },
    })
    return base
