"""`openquant gpu`: fused INT4 dequant-matmul benchmark on the B200.

The reference's report (openquant/fused_benchmark.py:37-120: FP32, FP16,
"old" decode-then-matmul and fused INT4 on (128, 2048) x (2048, 2048), g=32,
median of 40 event-timed calls, relative error vs the FP32 product), followed
by the decode and prefill shapes this build targets with GB/s, TFLOP/s and
% of the measured B200 roofline.
"""
import json
import os
from statistics import median

import numpy as np
import torch

from .group_benchmark import restore_groupwise_torch
from .groupwise import quantize_int4_groupwise
from .triton_int4 import int4_linear

__all__ = ["measure", "main"]

_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks():
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": float(p["hbm_gbs"]), "bf16_tflops": float(p["bf16_tflops"])}, "measured"
    except (OSError, ValueError, KeyError):
        return dict(_PEAKS), "fallback"


def measure(fn, repeats=40):
    """Median of `repeats` CUDA-event timings in ms after 10 warm-up calls
    (openquant/fused_benchmark.py:14-34)."""
    with torch.inference_mode():
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        samples = []
        for _ in range(repeats):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            out = fn()
            end.record()
            end.synchronize()
            samples.append(start.elapsed_time(end))
            del out
    return median(samples)


def _rel_err(y, ref):
    return (torch.linalg.vector_norm(y.float() - ref) / torch.linalg.vector_norm(ref) * 100).item()


def main():
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA GPU required")
    torch.set_float32_matmul_precision("highest")
    pk, src = peaks()
    rng = np.random.default_rng(42)
    weights = rng.normal(size=(2048, 2048)).astype(np.float32)
    inputs = rng.normal(size=(128, 2048)).astype(np.float32)
    x = torch.from_numpy(inputs).cuda()
    w = torch.from_numpy(weights).cuda()
    x16, w16 = x.half(), w.half()
    group_size = 32
    q = quantize_int4_groupwise(w, group_size)
    packed, scales = q.data, q.scales
    cases = [
        ("FP32", lambda: x @ w.T),
        ("FP16", lambda: x16 @ w16.T),
        ("Old INT4 decode", lambda: x @ restore_groupwise_torch(packed, scales, weights.shape, group_size).T),
        ("Fused B200 INT4", lambda: int4_linear(x16, packed, scales, weights.shape[0], group_size)),
    ]
    with torch.inference_mode():
        reference = x @ w.T
        torch.cuda.synchronize()
        print("\nOPENQUANT-B200 - FUSED GPU BENCHMARK")
        print("GPU:", torch.cuda.get_device_name())
        print("Shape: (128, 2048) x (2048, 2048)")
        print("INT4 group size:", group_size)
        print("-" * 58)
        for name, fn in cases:
            err = _rel_err(fn(), reference)
            print(f"{name:<22}{measure(fn):>9.4f} ms{err:>12.3f}% error")
    print("-" * 58)
    print(f"INT4 persistent storage: {(packed.numel() + scales.numel() * 4) / 1048576:.3f} MiB")
    print("FP32 persistent storage: 16.000 MiB")
    print("Timing excludes quantization and transfers.")

    print(f"\nB200 targets (roofline = {src} peaks: HBM {pk['hbm_gbs']:.0f} GB/s, bf16 {pk['bf16_tflops']:.0f} TFLOP/s)")
    print(f"{'shape (M, K, N, g)':<28}{'us':>10}{'GB/s':>10}{'TFLOP/s':>10}{'% roof':>8}")
    gen = torch.Generator(device="cuda").manual_seed(0)
    for m, k, n, dt in [(1, 4096, 4096, torch.float16), (1, 4096, 22016, torch.float16),
                        (16, 11008, 4096, torch.float16), (2048, 8192, 28672, torch.bfloat16)]:
        wq = quantize_int4_groupwise(torch.randn(n, k, device="cuda", generator=gen).mul_(0.02).to(dt), 128)
        xx = torch.randn(m, k, device="cuda", generator=gen).to(dt)
        out = torch.empty(m, n, device="cuda")
        ms = measure(lambda: int4_linear(xx, wq.data, wq.scales, n, 128, out=out), repeats=20)
        nbytes = n * k // 2 + n * (k // 128) * 4 + m * k * 2 + m * n * 4
        gbs, tf = nbytes / ms / 1e6, 2 * m * n * k / ms / 1e9
        frac = tf / pk["bf16_tflops"] if m >= 64 else gbs / pk["hbm_gbs"]
        print(f"{str((m, k, n, 128)):<28}{ms * 1e3:>10.1f}{gbs:>10.0f}{tf:>10.1f}{frac * 100:>7.1f}%")
        del wq, xx, out


if __name__ == "__main__":
    main()
