"""`openquant tune`: offline kernel / launch-shape search for int4_linear.

The reference searches Triton block shapes on one problem
(openquant/autotune.py:14-195: every config is checked against
x16 @ restored16.T with assert_close(rtol=atol=0.02), timed as the median of
30 calls, the fastest reported).  Here every candidate is a hand-written
sm_100a kernel and launch shape of oq_int4_linear -- the TMA-fed and
register-ring GEMVs, the tcgen05 GEMM and the CUDA-core kernel -- checked the
same way against the same reference, timed as back-to-back launches in a CUDA
graph over rotated weight copies (the way a decode step runs them), and the winner
per (M bucket, N, K, g) is written to openquant_b200/tile_table.json, which
int4_linear reads.
"""
import argparse
import json
from statistics import median

import torch

from . import _native as nat
from . import tile_table
from .group_benchmark import restore_groupwise_torch
from .groupwise import quantize_int4_groupwise

__all__ = ["CONFIGS", "SHAPES", "candidates", "time_gpu", "tune_shape", "main"]

# The reference's Triton (BM, BN, BK, warps) list (openquant/autotune.py:14-25).
# int4_linear still accepts these keywords; they select nothing here.
CONFIGS = [
    (16, 32, 32, 4), (16, 64, 64, 4), (32, 32, 64, 4), (32, 64, 64, 4), (32, 64, 128, 4),
    (32, 128, 64, 4), (64, 64, 64, 4), (64, 64, 128, 4), (64, 128, 64, 8), (64, 128, 128, 8),
]

# (M, K, N, g, x dtype): the reference's tuning problem, the Llama-2-7B decode
# layer set at M in {1, 4, 16} and the Llama-3-70B MLP prefill shapes.
SHAPES = [(128, 2048, 2048, 32, torch.float16)]
SHAPES += [(m, k, n, 128, torch.float16) for m in (1, 4, 16)
           for k, n in ((4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096))]
SHAPES += [(m, k, n, 128, torch.bfloat16) for m in (512, 2048) for k, n in ((8192, 28672), (28672, 8192))]


def candidates(m):
    """(name, kernel code, config) pairs worth trying at batch size m; the
    library's own shape rule ("auto") is one of them, so a table entry is
    never slower than leaving the shape out."""
    out = [("auto", 0, 0)]
    if m <= 64:
        shapes = [*range(1, 11), 12, 13] if m <= 16 else range(1, 8)
        # Above M = 16 the library's default is the exact weight rounding; a
        # table entry changes the launch shape, never the rounding.
        flag = nat.CONFIG_EXACT_ROUNDING if m > 16 else 0
        out += [(f"gemv:{c}", nat.KERNELS["gemv"], c | flag) for c in shapes]
    out.append(("tcgen05", nat.KERNELS["tcgen05"], 0))
    if m <= 256:
        out.append(("simt", nat.KERNELS["simt"], 0))
    return out


def time_gpu(fn, repetitions=30):
    """Median CUDA-event time in ms after 10 warm-up calls (autotune.py:28-49)."""
    with torch.inference_mode():
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(repetitions):
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record()
            fn()
            end.record()
            end.synchronize()
            times.append(start.elapsed_time(end))
    return median(times)


def time_stream(launch, copies, launches=64, repeats=3):
    """Per-launch time in ms of back-to-back launches captured in a CUDA graph,
    cycling through `copies` weight copies (so a decode GEMV streams its
    weights from HBM as it does between layers).  Decode kernels are
    latency-sized, so timing them one call at a time measures launch overhead
    rather than the kernel."""
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(min(copies, 4)):
            launch(i, stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(launches):
            launch(i % copies, torch.cuda.current_stream())
    graph.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(repeats):
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        end.record()
        end.synchronize()
        best = min(best, start.elapsed_time(end) / launches)
    del graph
    return best


def tune_shape(m, k, n, g, dtype, seed=0, verbose=True):
    """Returns (best name, kernel, config, ms) and prints every candidate."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02)
    q = quantize_int4_groupwise(w, g)
    del w
    x = torch.randn(m, k, device="cuda", generator=gen).to(dtype)
    with torch.inference_mode():
        wr = restore_groupwise_torch(q.data, q.scales, (n, k), g).to(dtype)
        reference = (x.float() @ wr.float().T)
        del wr
    y = torch.empty(m, n, device="cuda")
    code = nat.OQ_F16 if dtype == torch.float16 else nat.OQ_BF16
    lib = nat.load()
    layer_bytes = q.data.numel() + q.scales.numel() * 4
    copies = max(2, min(64, -(-300_000_000 // layer_bytes)))  # > 2x the 126 MB L2
    packs = [q.data] + [q.data.clone() for _ in range(copies - 1)]
    scs = [q.scales] + [q.scales.clone() for _ in range(copies - 1)]
    results, failures = [], []
    for name, kern, cfg in candidates(m):
        # Timed as a decode loop runs: the weights were quantized beforehand,
        # so every launch declares them static (the flag changes when they are
        # read, never the result, and is not part of the stored launch shape).
        def launch(i, stream):
            nat.check(lib.oq_int4_linear(nat.ptr(x), code, nat.ptr(packs[i]), nat.ptr(scs[i]), nat.ptr(y), m, n, k,
                                         g, kern, cfg | nat.CONFIG_STATIC_WEIGHTS, nat.ptr_of_stream(stream)))

        try:
            launch(0, torch.cuda.current_stream())
            torch.testing.assert_close(y, reference, rtol=0.02, atol=0.02)
            launches = 64 if m <= 64 else 8
            results.append((time_stream(launch, copies, launches=launches), name, kern, cfg))
        except (ValueError, RuntimeError, AssertionError) as exc:
            failures.append((name, str(exc).splitlines()[0][:120]))
    results.sort()
    if verbose:
        dt = "fp16" if dtype == torch.float16 else "bf16"
        print(f"\n(M={m}, K={k}, N={n}, g={g}, {dt})")
        for ms, name, _, _ in results:
            print(f"  {name:<10} {ms * 1e3:>10.1f} us")
        for name, why in failures:
            print(f"  {name:<10} {'-':>10}    not taken: {why}")
    if not results:
        return None
    ms, name, kern, cfg = results[0]
    return name, kern, cfg, ms


def main(argv=None):
    ap = argparse.ArgumentParser(prog="openquant tune", description=__doc__)
    ap.add_argument("--output", default=tile_table.TABLE_PATH, help="tile table to write")
    ap.add_argument("--quick", action="store_true", help="only the reference's tuning problem")
    args = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise RuntimeError("CUDA unavailable")
    nat.require_device()
    print("\nOPENQUANT-B200 - KERNEL TUNING")
    print("GPU:", torch.cuda.get_device_name(0))
    entries = []
    for (m, k, n, g, dtype) in (SHAPES[:1] if args.quick else SHAPES):
        best = tune_shape(m, k, n, g, dtype)
        if best is None:
            continue
        name, kern, cfg, ms = best
        print(f"  -> fastest verified: {name} ({ms * 1e3:.1f} us)")
        entries.append({"key": [tile_table.m_bucket(m), n, k, g], "kernel": kern, "split_k": cfg,
                        "name": name, "us": round(ms * 1e3, 2), "dtype": str(dtype).replace("torch.", "")})
    with open(args.output, "w") as f:
        json.dump({"device": torch.cuda.get_device_name(0), "entries": entries}, f, indent=1)
        f.write("\n")
    tile_table.reset()
    print(f"\nwrote {len(entries)} entries to {args.output}")
    return 0


if __name__ == "__main__":
    main()
