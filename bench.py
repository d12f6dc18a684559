#!/usr/bin/env python
"""Benchmark of the INT4 dequant-GEMV / GEMM path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (a "step"): one fused groupwise-INT4 dequant + matmul,
y[1,4096] = x[1,4096] . W^T, W 4096x4096 INT4 with group 128 and fp32
scales, fp16 activations ~ N(0,1), weights ~ N(0,0.02) -- the single-GPU
decode GEMV.  Each step reads a different one of 64 weight copies (572 MB,
4.5x the 126 MB L2), so every step streams its weights from HBM.  The K
steps run as CUDA-graph replays of back-to-back launches on one stream and
are timed with CUDA events; `value` is algorithmic bytes (8,937,472 per
step) / time, summed over ranks.  Under torchrun each rank streams its own
weight copies (weak scaling, no collective on the data path).

`e2e` times the same step through the public API (openquant.triton_int4.
int4_linear) with the activations copied from pinned host memory and the
output read back to the host every step.

`--impl reference` times the reference algorithm on the host cores (the
oracle's NumPy restatement of dequantize_int4_groupwise + fp16 rounding +
matmul, threaded over row blocks), each step a bounded row sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "INT4 dequant-GEMM: GB/s at M=1, TFLOP/s at M=2048, % of B200 roofline"
UNIT = "GB/s"
M, K, N, G = 1, 4096, 4096, 128
KP = ((K + G - 1) // G) * G
ALG_BYTES = N * KP // 2 + N * (KP // G) * 4 + M * K * 2 + M * N * 4  # 8,937,472
COPIES = 64
# e2e: host round trips timed on the wall clock, a fixed count whatever --steps is
# (a round trip is ~20 us, so 2000 of them take ~50 ms)
E2E_STEPS = 2000
COOL_DOWN_S = 1.0  # idle time before each prefill GEMM case is timed
ONE_GRAPH_MAX = 8192  # up to this many warm-up + timed launches, one graph each
L2_BYTES = 126 * 1024 * 1024
WORKLOAD = "int4_gemv_m1_k4096_n4096_g128_fp16"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def read_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return {k: float(p[k]) for k in FALLBACK_PEAKS}, "measured"
    except (OSError, ValueError, KeyError):
        return dict(FALLBACK_PEAKS), "fallback"


def read_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu
    summary (profiles/<name>.json), or None."""
    path = os.path.join(ROOT, "profiles", name + ".json")
    try:
        with open(path) as f:
            return float(json.load(f)["dram_bytes_per_launch"])
    except (OSError, ValueError, KeyError):
        return None


# ------------------------------------------------------------ clocks --


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples taken during the timed
    region (read-only queries)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, uuid):
        self.uuid = uuid
        self.proc = None
        self.file = None

    def start(self):
        try:
            self.file = tempfile.TemporaryFile(mode="w+")
            cmd = ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "20"]
            if self.uuid:
                cmd += ["-i", self.uuid]
            self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.count(",") >= 8]
        sm, smax, reasons = [], [], set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                smax.append(float(r[2]))
            except ValueError:
                continue
            for name, val in zip(self.NAMES, r[5:9]):
                if "Active" in val and "Not" not in val:
                    reasons.add(name)
        loaded = [s for s in sm if s > 0.5 * max(sm)] if sm else []
        return {
            "sm_mhz": statistics.median(loaded) if loaded else None,
            "sm_max_mhz": max(smax) if smax else None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


def headline_config(world):
    """`config` of the headline line, the same for both arms."""
    return {
        "workload": WORKLOAD,
        "m": M, "k": K, "n": N, "group_size": G,
        "weights": f"{COPIES} distinct INT4 copies rotated ({COPIES * ALG_BYTES / 1e6:.0f} MB > L2)",
        "l2": "inputs larger than L2 (weight-copy rotation), no flush",
        "launch": "CUDA graphs of back-to-back launches (programmatic dependent launch): the first of the W "
                  "warm-up launches eagerly (kernel set-up), then behind a device-side sleep (so the host's "
                  "submission is off the clock) the other W-1 warm-up launches, the start event, the K timed "
                  f"launches (one graph up to {ONE_GRAPH_MAX} launches), the end event",
        "static_weights": "weights quantized at setup and synchronized, so each launch streams them "
                          "while the previous one drains (OQ_CONFIG_STATIC_WEIGHTS); x and y stay ordered",
        "parallelism": f"dp{world} (each rank streams its own weight copies)",
    }


def summarize(line):
    """Compact figures of the headline and of every `also` line."""
    r3 = lambda v: None if v is None else round(float(v), 3)  # noqa: E731
    out = {"headline_gbs": r3(line["value"] / line["n_gpus"]), "headline_frac": r3(line["roofline"]["frac"]),
           "e2e_gbs": r3(line["e2e"]["value"])}
    for a in line.get("also", []):
        wl = a.get("workload", "")
        if wl.startswith("int4_gemv_llama2"):
            out["decode_set"] = {f"m{m}": {"gbs": r3(v["gbs"]), "frac": r3(v["frac"])} for m, v in a["by_m"].items()}
        elif wl.startswith("int4_gemm_llama3"):
            out["prefill_set"] = {c: {"tflops": r3(v["tflops"]), "frac": r3(v["frac"])}
                                  for c, v in a["by_case"].items()}
            if "gate_up_silu_m2048" in a:
                sc = a["gate_up_silu_m2048"]
                out["prefill_gate_up_silu_m2048"] = {"tflops": r3(sc["tflops"]), "frac": r3(sc["frac"]),
                                                     "speedup_vs_two_gemms": r3(sc["speedup_vs_two_gemms"])}
        elif wl.startswith("int4_gemm_m2048"):
            out["gemm_m2048"] = {"tflops": r3(a["value"]), "frac": r3(a["roofline"]["frac"])}
        elif wl.startswith("int8_gemm"):
            out["w8a8_m2048"] = {"tops": r3(a["value"]), "frac": r3(a["roofline"]["frac"])}
        elif wl.startswith("bulk_quant"):
            out["bulk_int4_g128"] = {"gbs": r3(a["value"]), "frac": r3(a["roofline"]["frac"])}
        elif wl.startswith("int4_linear_sharded"):
            out["sharded"] = {c: {k: r3(v[k]) for k in ("tflops", "us", "efficiency_vs_1gpu", "allgather_ms")
                                  if k in v} for c, v in a["by_case"].items()}
        elif wl.startswith("int4_gemv_m1_k4096_n4096_g128_fp16_scales"):
            out["gemv_fp16_scales"] = {"gbs": r3(a["value"]), "frac": r3(a["roofline"]["frac"])}
        elif wl.startswith("cpu_path_1024"):
            out["cpu_path_1024"] = {f: {"gpu_ms": r3(v["gpu_ms"]), "cpu_ms": r3(v["cpu_ms"]),
                                        "rel_weight_err": r3(v["rel_weight_err"])} for f, v in a["formats"].items()}
    return out


# ---------------------------------------------------------- CPU side --


_CPU_LAYER = {}


def _cpu_layer():
    """The host copy of one INT4 layer (quantized once by the oracle)."""
    if not _CPU_LAYER:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oq_oracle as orc

        rng = np.random.default_rng(7)
        w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
        data, scales = orc.quantize_int4_groupwise(w, G)
        x = orc.round_to_dtype(rng.normal(size=(M, K)).astype(np.float32), "f16")
        _CPU_LAYER.update(orc=orc, data=data.reshape(N, KP // 2), scales=scales, x=x)
    return _CPU_LAYER


def cpu_gemv_sample(rows, threads):
    """One reference-algorithm step on the host: dequantize `rows` rows of
    the INT4 layer, round them to fp16, multiply with x (fp32 BLAS).
    Returns (seconds, algorithmic bytes of the sample)."""
    layer = _cpu_layer()
    orc, data2, scales, x = layer["orc"], layer["data"], layer["scales"], layer["x"]

    def block(r0, r1):
        wd = orc.dequantize_int4_groupwise(data2[r0:r1].reshape(-1), scales[r0:r1], (r1 - r0, K), G)
        return x @ orc.round_to_dtype(wd, "f16").T

    from threadpoolctl import threadpool_limits

    # One BLAS thread per worker thread: the row blocks already use every core.
    with threadpool_limits(limits=1):
        t0 = time.perf_counter()
        y = np.concatenate(orc.threaded_rows(block, rows, threads=threads, min_rows=16), axis=1)
        dt = time.perf_counter() - t0
    assert y.shape == (M, rows)
    sample_bytes = rows * KP // 2 + rows * (KP // G) * 4 + M * K * 2 + M * rows * 4
    return dt, sample_bytes


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_baseline(budget_s=10.0):
    threads = cpu_threads()
    cpu_gemv_sample(N, threads)  # warm-up
    times, nbytes = [], 0
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end and len(times) < 50:
        dt, nbytes = cpu_gemv_sample(N, threads)
        times.append(dt)
    med = statistics.median(times)
    return {
        "value": nbytes / med / 1e9,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{len(times)} full {N}x{K} g={G} layers (dequantize + fp16 round + x@W^T, NumPy/OpenBLAS, "
                  f"{threads} threads over row blocks, 1 BLAS thread each), median {med * 1e3:.1f} ms",
    }


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = cpu_threads()
    total = args.steps + args.warmup
    budget = 120.0  # seconds for the whole run
    dt_full, _ = cpu_gemv_sample(N, threads)
    per_step = budget / max(total, 1)
    rows = int(max(16, min(N, N * per_step / max(dt_full, 1e-6))))
    for _ in range(args.warmup):
        cpu_gemv_sample(rows, threads)
    secs, nbytes = 0.0, 0
    for _ in range(args.steps):
        dt, b = cpu_gemv_sample(rows, threads)
        secs += dt
        nbytes += b
    value = nbytes / secs / 1e9
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": headline_config(int(os.environ.get("WORLD_SIZE", "1"))),
        "cpu_baseline": {
            "value": value,
            "unit": UNIT,
            "cores": threads,
            "kind": "port",
            "sample": f"{rows} of {N} rows of the layer per step (NumPy restatement of the reference's "
                      f"dequantize_int4_groupwise + fp16 rounding + matmul, {threads} threads)",
        },
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------- GPU side --


def measure_gemm(dev, peaks, steps=10, warmup=3):
    """TFLOP/s of the prefill GEMM at M = 2048, (K, N) = (8192, 28672) (the
    Llama-3-70B gate/up projection), bf16 x, group 128, two weight copies
    (2 x 117 MB packed, beyond L2) alternated; CUDA-graph replay, CUDA events."""
    import ctypes

    import torch

    from openquant_b200 import _native as nat
    from openquant_b200.groupwise import quantize_int4_groupwise

    lib = nat.load()
    m, k, n, g = 2048, 8192, 28672, 128
    gen = torch.Generator(device=dev).manual_seed(77)
    w = torch.randn(n, k, generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
    q = quantize_int4_groupwise(w, g)
    del w
    packs, scs = [q.data, q.data.clone()], [q.scales, q.scales.clone()]
    x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
    y = torch.empty(m, n, device=dev)
    ws_bytes = lib.oq_int4_linear_workspace_bytes(m, n, k, g, 0, 0)
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()  # inputs made on the default stream, launches on `stream`

    def launch(count, h):
        for i in range(count):
            st = lib.oq_int4_linear_ws(ctypes.c_void_p(x.data_ptr()), nat.OQ_BF16,
                                       ctypes.c_void_p(packs[i % 2].data_ptr()), ctypes.c_void_p(scs[i % 2].data_ptr()),
                                       ctypes.c_void_p(y.data_ptr()), nat.OQ_F32, None, m, n, k, g, 0, 0,
                                       ctypes.c_void_p(ws.data_ptr()), ws_bytes, h)
            if st != 0:
                raise RuntimeError(nat.last_error())

    with torch.cuda.stream(stream):
        launch(warmup, ctypes.c_void_p(stream.cuda_stream))
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch(steps, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    graph.replay()
    torch.cuda.synchronize()
    time.sleep(COOL_DOWN_S)
    ms = _device_timed(stream, graph.replay, steps)
    tflops = 2.0 * m * n * k / (ms / 1e3) / 1e12
    # spot check against the exactly-rounded weights on sampled columns
    from oq_oracle import dequantize_int4_groupwise as deq, round_to_dtype

    rows = torch.arange(0, n, 1021, device=dev)
    wr = round_to_dtype(deq(q.data.view(n, k // 2)[rows].cpu().numpy().reshape(-1), q.scales[rows].cpu().numpy(),
                            (len(rows), k), g), "bf16")
    ref = x.double() @ torch.from_numpy(wr).to(dev).double().T
    rel = ((y[:, rows].double() - ref).norm() / ref.norm()).item()
    mab = (y[:, rows].double() - ref).abs().max().item()
    assert rel <= 1e-3 and mab <= 2e-2, (rel, mab)
    del graph
    return {
        "metric": "INT4 dequant-GEMM TFLOP/s at M=2048",
        "workload": "int4_gemm_m2048_k8192_n28672_g128_bf16",
        "value": tflops,
        "unit": "TFLOP/s",
        "ms_per_step": ms,
        "steps": steps,
        "roofline": {
            "bound": "tensor",
            "achieved": tflops,
            "peak": peaks["bf16_tflops"],
            "unit": "TFLOP/s",
            "frac": tflops / peaks["bf16_tflops"],
            "frac_of_sustained": tflops / peaks["bf16_tflops_sustained"],
            "traffic": read_traffic("gemm_m2048_k8192_n28672_g128"),
            "algorithmic_flops_per_launch": 2 * m * n * k,
        },
        "gpu_launches": steps,
        "check_rel_l2": rel,
        "check_max_abs": mab,
    }


PREFILL_SHAPES = [("gate_up", 8192, 28672), ("down", 28672, 8192)]


def measure_prefill_set(dev, peaks, ms_=(512, 2048, 8192), steps=10, warmup=3):
    """TFLOP/s of the prefill GEMM on the Llama-3-70B MLP shapes (gate/up
    8192->28672, down 28672->8192), bf16 x ~ N(0,1), weights ~ N(0,0.02)
    group 128, at M = 512, 2048 and 8192; two weight copies alternate (each
    beyond L2), CUDA-graph replay, CUDA events.  Each case is checked on
    sampled weight rows against the exactly-rounded weights."""
    import ctypes

    import torch

    from oq_oracle import dequantize_int4_groupwise as deq, round_to_dtype
    from openquant_b200 import _native as nat
    from openquant_b200.groupwise import quantize_int4_groupwise

    lib = nat.load()
    g = 128
    stream = torch.cuda.Stream(device=dev)
    cases, rel_worst, abs_worst, launches = {}, 0.0, 0.0, 0
    for si, (name, k, n) in enumerate(PREFILL_SHAPES):
        gen = torch.Generator(device=dev).manual_seed(700 + si)
        w = torch.randn(n, k, generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
        q = quantize_int4_groupwise(w, g)
        del w
        packs, scs = [q.data, q.data.clone()], [q.scales, q.scales.clone()]
        rows = torch.arange(0, n, 1021, device=dev)
        wr = torch.from_numpy(round_to_dtype(deq(q.data.view(n, k // 2)[rows].cpu().numpy().reshape(-1),
                                                 q.scales[rows].cpu().numpy(), (len(rows), k), g), "bf16")).to(dev)
        for m in ms_:
            x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
            y = torch.empty(m, n, device=dev)
            ws_bytes = lib.oq_int4_linear_workspace_bytes(m, n, k, g, 0, 0)
            ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
            torch.cuda.synchronize()  # inputs made on the default stream, launches on `stream`

            def launch(count, h):
                for i in range(count):
                    st = lib.oq_int4_linear_ws(ctypes.c_void_p(x.data_ptr()), nat.OQ_BF16,
                                               ctypes.c_void_p(packs[i % 2].data_ptr()),
                                               ctypes.c_void_p(scs[i % 2].data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                               nat.OQ_F32, None, m, n, k, g, 0, 0, ctypes.c_void_p(ws.data_ptr()),
                                               ws_bytes, h)
                    if st != 0:
                        raise RuntimeError(nat.last_error())

            with torch.cuda.stream(stream):
                launch(warmup, ctypes.c_void_p(stream.cuda_stream))
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                launch(steps, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            graph.replay()
            torch.cuda.synchronize()
            time.sleep(COOL_DOWN_S)  # the previous case's power draw must not cap this one's clocks
            ms = _device_timed(stream, graph.replay, steps)
            del graph
            launches += warmup + 2 * steps
            tflops = 2.0 * m * n * k / (ms / 1e3) / 1e12
            ref = x.double() @ wr.double().T
            rel = ((y[:, rows].double() - ref).norm() / ref.norm()).item()
            mab = (y[:, rows].double() - ref).abs().max().item()
            assert rel <= 1e-3 and mab <= 2e-2, (name, m, rel, mab)
            rel_worst, abs_worst = max(rel_worst, rel), max(abs_worst, mab)
            cases[f"{name}_m{m}_k{k}_n{n}"] = {"ms": ms, "tflops": tflops, "frac": tflops / peaks["bf16_tflops"],
                                              "frac_of_sustained": tflops / peaks["bf16_tflops_sustained"],
                                              "split": ws_bytes > 0}
            del x, y, ws
        del packs, scs, q
        torch.cuda.empty_cache()
    silu_case = _measure_prefill_silu(dev, peaks, stream, steps, warmup)
    launches += silu_case.pop("launches")
    return {
        "metric": "INT4 dequant-GEMM TFLOP/s over the Llama-3-70B MLP prefill set",
        "workload": "int4_gemm_llama3_70b_mlp_g128_bf16",
        "value": cases[f"gate_up_m2048_k8192_n28672"]["tflops"] if 2048 in ms_ else None,
        "unit": "TFLOP/s",
        "value_is": "gate/up at M=2048; every (shape, M) case in by_case",
        "by_case": cases,
        "gate_up_silu_m2048": silu_case,
        "timing": f"each case after {COOL_DOWN_S} s idle: a kernel timed alone (burst peak), not under the power "
                  "cap the previous case's GEMMs leave behind",
        "gpu_launches": launches,
        "check_rel_l2": rel_worst,
        "check_max_abs": abs_worst,
    }


def _measure_prefill_silu(dev, peaks, stream, steps, warmup, m=2048, k=8192, n=28672, g=128):
    """The Llama-3-70B MLP's gate and up projections fused (silu_gate): the
    [gate; up] stack of 2 x 28672 rows, K = 8192, M = 2048 bf16 x, one tcgen05
    GEMM whose epilogue writes silu(gate) * up (28672 features), against the
    two plain GEMMs it replaces (gate, up: two fp32 outputs, no silu pass).
    Sampled columns must equal silu(gate) * up of the two GEMMs within a few
    fp32 ulp."""
    import ctypes

    import torch

    from openquant_b200 import _native as nat
    from openquant_b200.groupwise import quantize_int4_groupwise

    lib = nat.load()
    gen = torch.Generator(device=dev).manual_seed(750)
    w = torch.randn(2 * n, k, generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
    q = quantize_int4_groupwise(w, g)
    del w
    x = torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16)
    half = q.data.numel() // 2
    y = torch.empty(m, n, device=dev)
    yg, yu = torch.empty(m, n, device=dev), torch.empty(m, n, device=dev)
    tc = nat.KERNELS["tcgen05"]

    def call(packed, scales, out, cols, cfg, h):
        st = lib.oq_int4_linear(ctypes.c_void_p(x.data_ptr()), nat.OQ_BF16, ctypes.c_void_p(packed.data_ptr()),
                                ctypes.c_void_p(scales.data_ptr()), ctypes.c_void_p(out.data_ptr()), m, cols, k, g,
                                tc, cfg, h)
        if st != 0:
            raise RuntimeError(nat.last_error())

    def fused(count, h):
        for _ in range(count):
            call(q.data, q.scales, y, n, nat.CONFIG_SILU_GATE, h)

    def separate(count, h):
        for _ in range(count):
            call(q.data[:half], q.scales[:n], yg, n, 0, h)
            call(q.data[half:], q.scales[n:], yu, n, 0, h)

    torch.cuda.synchronize()
    out = {"launches": 0}
    for name, body in (("fused", fused), ("two_gemms", separate)):
        with torch.cuda.stream(stream):
            body(warmup, ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            body(steps, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        graph.replay()
        torch.cuda.synchronize()
        time.sleep(COOL_DOWN_S)
        out[name + "_ms"] = _device_timed(stream, graph.replay, steps)
        del graph
        out["launches"] += (warmup + 2 * steps) * (1 if name == "fused" else 2)
    cols = torch.arange(0, n, 997, device=dev)
    gsel, usel = yg[:, cols].double(), yu[:, cols].double()
    ref = gsel * torch.sigmoid(gsel) * usel
    err = (y[:, cols].double() - ref).abs()
    assert float((err - 2e-6 * ref.abs()).max()) <= 1e-6, float(err.max())
    flops = 2.0 * m * (2 * n) * k
    out["tflops"] = flops / (out["fused_ms"] / 1e3) / 1e12
    out["frac"] = out["tflops"] / peaks["bf16_tflops"]
    out["speedup_vs_two_gemms"] = out["two_gemms_ms"] / out["fused_ms"]
    out["check"] = "sampled columns equal silu(gate) * up of the two plain GEMMs within 2e-6 relative + 1e-6"
    return out


DECODE_LAYERS = [("qkv", 4096, 12288), ("o_proj", 4096, 4096), ("gate_up", 4096, 22016), ("down", 11008, 4096)]


def measure_decode_layers(dev, peaks, ms_=(1, 4, 16), sets=3, steps=200, warmup=20):
    """GB/s of the decode GEMV over the Llama-2-7B layer set (fused QKV
    4096->12288, O 4096->4096, fused gate/up 4096->22016, down 11008->4096),
    group 128, fp16 x ~ N(0,1), weights ~ N(0,0.02) seeded per layer, at
    M = 1, 4 and 16.  A step runs the four layers back to back through
    oq_int4_linear (automatic kernel choice, static weights); `sets` copies
    of the whole layer set (3 x 107 MB, beyond L2) are rotated.  Each layer
    is also timed alone (a graph of its own launches over the copies)."""
    import ctypes

    import torch

    from openquant_b200 import _native as nat
    from openquant_b200 import tile_table
    from openquant_b200.groupwise import Groupwise4, dequantize_int4_groupwise, quantize_int4_groupwise

    lib = nat.load()
    g = 128
    layers = []  # per layer: (name, k, n, [(packed, scales)] * sets, bytes of weights + scales)
    for li, (name, k, n) in enumerate(DECODE_LAYERS):
        copies = []
        for s in range(sets):
            gen = torch.Generator(device=dev).manual_seed(500 + 10 * li + s)
            w = torch.randn(n, k, generator=gen, device=dev).mul_(0.02).half()
            q = quantize_int4_groupwise(w, g)
            del w
            copies.append((q.data, q.scales))
        layers.append((name, k, n, copies, n * k // 2 + n * (k // g) * 4))
    stream = torch.cuda.Stream(device=dev)
    out = {}
    rel_worst, abs_worst = 0.0, 0.0
    launches = 0
    for m in ms_:
        gen = torch.Generator(device=dev).manual_seed(900 + m)
        xs = [torch.randn(m, k, generator=gen, device=dev).half() for (_, k, _, _, _) in layers]
        ys = [torch.empty(m, n, device=dev) for (_, _, n, _, _) in layers]
        torch.cuda.synchronize()  # inputs made on the default stream, launches on `stream`
        # the launch shape int4_linear / Int4Linear choose: the tuned table's
        # entry for (M bucket, N, K, g), else the library's automatic choice
        choice = [tile_table.lookup(m, n, k, g) for (_, k, n, _, _) in layers]
        calls = [[(ctypes.c_void_p(xs[li].data_ptr()), nat.OQ_F16, ctypes.c_void_p(p.data_ptr()),
                   ctypes.c_void_p(sc.data_ptr()), ctypes.c_void_p(ys[li].data_ptr()), m, n, k, g, choice[li][0],
                   choice[li][1] | nat.CONFIG_STATIC_WEIGHTS) for (p, sc) in copies]
                 for li, (_, k, n, copies, _) in enumerate(layers)]
        io = [m * k * 2 + m * n * 4 for (_, k, n, _, _) in layers]

        def timed(seq):
            """µs for the launch sequence `seq` (oq_int4_linear argument
            tuples) replayed as one CUDA graph, after an eager warm-up."""
            def run(h, items):
                for a in items:
                    if lib.oq_int4_linear(*a, h) != 0:
                        raise RuntimeError(nat.last_error())
            with torch.cuda.stream(stream):
                run(ctypes.c_void_p(stream.cuda_stream), seq[:warmup])
            stream.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                run(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), seq)
            graph.replay()
            torch.cuda.synchronize()
            ms = _device_timed(stream, graph.replay, 1)
            del graph
            return ms * 1e3

        step_seq = [calls[li][s % sets] for s in range(steps) for li in range(len(layers))]
        step_us = timed(step_seq) / steps
        launches += len(step_seq)
        step_bytes = sum(b for (*_, b) in layers) + sum(io)
        per_layer = {}
        for li, (name, k, n, _, wb) in enumerate(layers):
            us = timed([calls[li][s % sets] for s in range(steps)]) / steps
            launches += steps
            gbs = (wb + io[li]) / us / 1e3
            per_layer[f"{name}_{k}x{n}"] = {"us": us, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"]}
        # spot check: the O projection (weight copy 0, run once more) against
        # the reference's dequantise-then-matmul
        with torch.cuda.stream(stream):
            nat.check(lib.oq_int4_linear(*calls[1][0], ctypes.c_void_p(stream.cuda_stream)))
        stream.synchronize()
        p, sc = layers[1][3][0]
        wref = dequantize_int4_groupwise(Groupwise4(p, sc, (4096, 4096), g)).half().double()
        yref = xs[1].double() @ wref.T
        rel = ((ys[1].double() - yref).norm() / yref.norm()).item()
        mab = (ys[1].double() - yref).abs().max().item()
        assert rel <= 1e-3 and mab <= 2e-2, (rel, mab)
        rel_worst, abs_worst = max(rel_worst, rel), max(abs_worst, mab)
        gbs = step_bytes / step_us / 1e3
        out[str(m)] = {"us_per_step": step_us, "gbs": gbs, "frac": gbs / peaks["hbm_gbs"], "layers": per_layer}
    del layers
    return {
        "metric": "INT4 decode GEMV GB/s over the Llama-2-7B layer set (QKV, O, gate/up, down)",
        "workload": "int4_gemv_llama2_7b_layers_g128_fp16",
        "value": out["1"]["gbs"] if "1" in out else None,
        "unit": "GB/s",
        "value_is": "M=1, one step = the four layers back to back; per-M and per-layer figures in by_m",
        "by_m": out,
        "l2": f"{sets} copies of the layer set rotated (> L2)",
        "launch": "CUDA graph of back-to-back launches (programmatic dependent launch), static weights",
        "gpu_launches": launches,
        "check_rel_l2": rel_worst,
        "check_max_abs": abs_worst,
    }


def measure_w8a8(dev, peaks, steps=10, warmup=3):
    """TOPS of the W8A8 GEMM (per-token INT8 x, per-row INT8 W, tcgen05
    kind::i8) at M = 2048, (K, N) = (8192, 28672), two weight copies
    alternated (2 x 235 MB, beyond L2); CUDA-graph replay, CUDA events.  The
    roofline peak is twice the measured bf16 GEMM rate (the B200's dense INT8
    rate is twice its BF16 rate; no INT8 peak is measured)."""
    import ctypes

    import torch

    from openquant_b200 import _native as nat

    lib = nat.load()
    m, k, n = 2048, 8192, 28672
    gen = torch.Generator(device=dev).manual_seed(81)
    qws = [torch.randint(-127, 128, (n, k), generator=gen, device=dev, dtype=torch.int8) for _ in range(2)]
    sw = torch.rand(n, generator=gen, device=dev) * 0.01 + 1e-3
    qx = torch.randint(-127, 128, (m, k), generator=gen, device=dev, dtype=torch.int8)
    sx = torch.rand(m, generator=gen, device=dev) * 0.01 + 1e-3
    y = torch.empty(m, n, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()  # inputs made on the default stream, launches on `stream`

    def launch(count, h):
        for i in range(count):
            st = lib.oq_int8_gemm(ctypes.c_void_p(qx.data_ptr()), ctypes.c_void_p(sx.data_ptr()),
                                  ctypes.c_void_p(qws[i % 2].data_ptr()), ctypes.c_void_p(sw.data_ptr()),
                                  ctypes.c_void_p(y.data_ptr()), m, n, k, h)
            if st != 0:
                raise RuntimeError(nat.last_error())

    with torch.cuda.stream(stream):
        launch(warmup, ctypes.c_void_p(stream.cuda_stream))
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch(steps, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    graph.replay()
    torch.cuda.synchronize()
    ms = _device_timed(stream, graph.replay, steps)
    del graph
    tops = 2.0 * m * n * k / (ms / 1e3) / 1e12
    # exact check on sampled columns: the int32 sums are exact, the epilogue rounds three times
    cols = torch.arange(0, n, 1021, device=dev)
    w = qws[(steps - 1) % 2]
    ref = (qx.double() @ w[cols].double().T) * sx.double()[:, None] * sw[cols].double()[None, :]
    rel = float(((y[:, cols].double() - ref).abs() / ref.abs().clamp_min(1e-30)).max())
    assert rel < 4e-7, rel
    peak = 2.0 * peaks["bf16_tflops"]
    return {
        "metric": "W8A8 GEMM TOPS at M=2048 (per-token INT8 x, per-row INT8 W)",
        "workload": "int8_gemm_m2048_k8192_n28672",
        "value": tops,
        "unit": "TOPS",
        "ms_per_step": ms,
        "steps": steps,
        "roofline": {"bound": "tensor", "achieved": tops, "peak": peak, "unit": "TOPS", "frac": tops / peak,
                     "peak_source": "2 x measured bf16 GEMM TFLOP/s (dense INT8 rate is twice BF16)",
                     "algorithmic_ops_per_launch": 2 * m * n * k},
        "gpu_launches": steps,
        "check_max_rel_err": rel,
    }


def measure_gemv_fp16_scales(dev, peaks, steps=2000, warmup=100):
    """The headline GEMV (M=1, K=N=4096, g=128, fp16 x) with one fp16 scale
    per group (oq_int4_linear_f16s; the reference's format is fp32 scales):
    the same packed weights, scales rounded to fp16, 64 copies rotated, static
    weights, one CUDA graph of `steps` launches behind a device sleep, CUDA
    events.  Checked against the oracle with the fp16 scales widened to fp32
    (rel-L2 <= 1e-3, max-abs <= 2e-2)."""
    import ctypes

    import torch

    from oq_oracle import int4_linear as orc_linear
    from openquant_b200 import _native as nat
    from openquant_b200.groupwise import quantize_int4_groupwise

    lib = nat.load()
    gen = torch.Generator(device=dev).manual_seed(4242)
    packs, s16s = [], []
    for _ in range(COPIES):
        q = quantize_int4_groupwise(torch.randn(N, K, generator=gen, device=dev).mul_(0.02).half(), G)
        packs.append(q.data)
        s16s.append(q.scales.half())
    x = torch.randn(M, K, generator=gen, device=dev).half()
    y = torch.empty(M, N, device=dev)
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()

    def launch(count, h, first=0):
        for i in range(first, first + count):
            st = lib.oq_int4_linear_f16s(ctypes.c_void_p(x.data_ptr()), nat.OQ_F16,
                                         ctypes.c_void_p(packs[i % COPIES].data_ptr()),
                                         ctypes.c_void_p(s16s[i % COPIES].data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                         nat.OQ_F32, None, M, N, K, G, nat.CONFIG_STATIC_WEIGHTS, h)
            if st != 0:
                raise RuntimeError(nat.last_error())

    with torch.cuda.stream(stream):
        launch(warmup, ctypes.c_void_p(stream.cuda_stream))
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        launch(steps, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), first=warmup)
    upload_graph(graph, stream)
    torch.cuda.synchronize()
    ms = _device_timed(stream, graph.replay, steps)
    del graph
    nbytes = N * KP // 2 + N * (KP // G) * 2 + M * K * 2 + M * N * 4
    gbs = nbytes / (ms / 1e3) / 1e9
    # parity: the last launch's copy against the oracle with the scales widened to fp32
    last = (warmup + steps - 1) % COPIES
    ref = orc_linear(x.float().cpu().numpy(), packs[last].cpu().numpy(), s16s[last].float().cpu().numpy(), N, G,
                     x_dtype="f16")
    err = y.double().cpu().numpy() - ref
    rel = float(np.linalg.norm(err) / np.linalg.norm(ref))
    mab = float(np.abs(err).max())
    assert rel <= 1e-3 and mab <= 2e-2, (rel, mab)
    return {
        "metric": "INT4 GEMV GB/s at M=1, K=N=4096, g=128, one fp16 scale per group (variant)",
        "workload": "int4_gemv_m1_k4096_n4096_g128_fp16_scales",
        "value": gbs,
        "unit": "GB/s",
        "ms_per_step": ms,
        "steps": steps,
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "algorithmic_bytes_per_launch": nbytes},
        "vs_fp32_scales": "the headline line: same weights format but fp32 scales (8,937,472 B per launch)",
        "gpu_launches": warmup + steps,
        "check_rel_l2": rel,
        "check_max_abs": mab,
    }


def measure_cpu_path_1024(dev, peaks, steps=50, warmup=5):
    """The reference's CPU NumPy case (quantization.py:14-82, benchmark.py:7-38)
    on the GPU: W 1024x1024 fp32 ~ N(0, 0.02) and x 16x1024 ~ N(0, 1) from
    np.random.default_rng(0); per format (INT8 per-row, packed INT4 per-row)
    one step = quantize -> dequantize -> x @ W_hat^T (the matmul in fp32,
    TF32 off), CUDA-graph replays timed with CUDA events.  The quantized bytes
    and scales must equal the oracle's; the reported errors are the
    reference's weight error ||W_hat - W|| / ||W|| and the output's relative
    error against x @ W^T.  The CPU side times the oracle's NumPy restatement of
    the same three steps on the host (NumPy ufuncs on one core, the matmul on
    the BLAS threads)."""
    import ctypes

    import torch

    from oq_oracle import dequantize as odeq, quantize as oquant
    from openquant_b200 import _native as nat

    lib = nat.load()
    rng = np.random.default_rng(0)
    w = rng.normal(0, 0.02, (1024, 1024)).astype(np.float32)
    x = rng.normal(0, 1, (16, 1024)).astype(np.float32)
    n, k = w.shape
    wt, xt = torch.from_numpy(w).to(dev), torch.from_numpy(x).to(dev)
    yref = x.astype(np.float64) @ w.astype(np.float64).T
    stream = torch.cuda.Stream(device=dev)
    tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    formats, launches = {}, 0
    try:
        for bits in (8, 4):
            q = torch.empty(n * k if bits == 8 else (n * k + 1) // 2, dtype=torch.uint8, device=dev)
            sc = torch.empty(n, device=dev)
            wd = torch.empty(n, k, device=dev)
            y = torch.empty(16, n, device=dev)
            torch.cuda.synchronize()

            def step(h):
                if bits == 8:
                    nat.check(lib.oq_quant_int8_rowwise(ctypes.c_void_p(wt.data_ptr()), nat.OQ_F32, n, k,
                                                        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()), h))
                    nat.check(lib.oq_dequant_int8_rowwise(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                                          n, k, ctypes.c_void_p(wd.data_ptr()), h))
                else:
                    nat.check(lib.oq_quant_int4_rowwise(ctypes.c_void_p(wt.data_ptr()), nat.OQ_F32, n, k,
                                                        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()), h))
                    nat.check(lib.oq_dequant_int4_rowwise(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                                          n, k, ctypes.c_void_p(wd.data_ptr()), h))
                torch.matmul(xt, wd.T, out=y)

            with torch.cuda.stream(stream):
                for _ in range(warmup):
                    step(ctypes.c_void_p(stream.cuda_stream))
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for _ in range(steps):
                        step(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            torch.cuda.synchronize()
            gpu_ms = _device_timed(stream, graph.replay, steps)
            del graph
            launches += 3 * (warmup + steps)
            d_ref, s_ref = oquant(w, bits)
            got = q.cpu().numpy()
            assert np.array_equal(got.view(np.int8) if bits == 8 else got, d_ref.reshape(-1)), bits
            assert np.array_equal(sc.cpu().numpy().view(np.uint32), s_ref.reshape(-1).view(np.uint32)), bits
            wd_np = wd.cpu().numpy()
            assert np.array_equal(wd_np.view(np.uint32), odeq(d_ref, s_ref, bits, (n, k)).view(np.uint32)), bits
            rel_w = float(np.linalg.norm(wd_np - w) / np.linalg.norm(w))
            rel_y = float(np.linalg.norm(y.cpu().numpy() - yref) / np.linalg.norm(yref))
            # the same three steps on the host (oracle restatement of the reference's NumPy code)
            times = []
            for _ in range(7):
                t0 = time.perf_counter()
                d_, s_ = oquant(w, bits)
                _ = x @ odeq(d_, s_, bits, (n, k)).T
                times.append(time.perf_counter() - t0)
            cpu_ms = statistics.median(times) * 1e3
            formats[f"int{bits}_rowwise"] = {"gpu_ms": gpu_ms, "gpu_mweights_s": n * k / gpu_ms / 1e3,
                                             "cpu_ms": cpu_ms, "cpu_mweights_s": n * k / cpu_ms / 1e3,
                                             "rel_weight_err": rel_w, "rel_output_err": rel_y}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = tf32
    head = formats["int4_rowwise"]
    return {
        "metric": "CPU-path case on the GPU: quantize + dequantize + x[16,1024] @ W_hat^T per second, "
                  "W 1024x1024 fp32 N(0,0.02) seed 0",
        "workload": "cpu_path_1024x1024_int8_int4",
        "value": head["gpu_mweights_s"],
        "unit": "Mweights/s",
        "value_is": "INT4 per-row; INT8 and INT4 in formats",
        "formats": formats,
        "gpu_launches": launches,
        "launch": "CUDA graph of the three steps (quantize and dequantize kernels, cuBLAS fp32 matmul, TF32 off)",
        "check": "quantized bytes, scales and dequantized weights bit-exact vs the oracle",
        "cpu_baseline": {"value": head["cpu_mweights_s"], "unit": "Mweights/s", "cores": 1, "kind": "port",
                         "sample": "the whole case, median of 7 (NumPy ufuncs on one core; the 16x1024x1024 "
                                   "matmul on the BLAS threads)"},
    }


# One Llama-3-70B decoder layer: (rows = out features, cols = in features)
# of its seven projection matrices; 855,638,016 weights.
BULK_SHAPES = [("q_proj", 8192, 8192), ("k_proj", 1024, 8192), ("v_proj", 1024, 8192), ("o_proj", 8192, 8192),
               ("gate_proj", 28672, 8192), ("up_proj", 28672, 8192), ("down_proj", 8192, 28672)]
BULK_LAYERS = 80
BULK_POOL = 4
BULK_FORMATS = [("int4_g128", 128), ("int4_g64", 64), ("int4_g32", 32), ("int8_rowwise", 0)]


def _bulk_layer(dev, layer):
    """Layer `layer`'s seven bf16 matrices, generated on the GPU from a
    per-layer seed: N(0, 0.02) with 0.1 % of the entries set to +-0.2."""
    import torch

    gen = torch.Generator(device=dev).manual_seed(9000 + layer)
    mats = []
    for _, n, k in BULK_SHAPES:
        w = torch.empty(n, k, device=dev).normal_(0.0, 0.02, generator=gen)
        idx = torch.randint(0, n * k, (n * k // 1000,), device=dev, generator=gen)
        w.view(-1)[idx] = torch.randint(0, 2, (idx.numel(),), device=dev, generator=gen).float() * 0.4 - 0.2
        mats.append(w.to(torch.bfloat16))
        del w
    return mats


def _bulk_bytes(fmt_g, layers):
    w = layers * sum(n * k for _, n, k in BULK_SHAPES)
    if fmt_g:
        return w, w * 2 + w // 2 + (w // fmt_g) * 4
    rows = layers * sum(n for _, n, _ in BULK_SHAPES)
    return w, w * 2 + w + rows * 4


def cpu_bulk_sample(rows=2048, k=8192, g=128):
    """The oracle's groupwise quantizer (NumPy restatement of
    quantize_int4_groupwise) on `rows` rows of a bf16-valued matrix, threaded
    over row blocks: (weights / s, threads)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oq_oracle as orc

    rng = np.random.default_rng(3)
    w = orc.round_to_dtype(rng.normal(0, 0.02, (rows, k)).astype(np.float32), "bf16")
    threads = cpu_threads()
    orc.threaded_rows(lambda a, b: orc.quantize_int4_groupwise(w[a:b], g), 64, threads=threads, min_rows=16)
    t0 = time.perf_counter()
    orc.threaded_rows(lambda a, b: orc.quantize_int4_groupwise(w[a:b], g), rows, threads=threads, min_rows=16)
    return rows * k / (time.perf_counter() - t0), threads


def measure_bulk_quant(dev, world, rank, peaks, layers=BULK_LAYERS):
    """Bulk quantization of a Llama-3-70B stack (80 layers x 7 matrices,
    68,451,041,280 bf16 weights) into each format: INT4 groupwise with g =
    128, 64, 32 and INT8 per-row.  Layers are assigned round-robin to the
    ranks (no collective on the data path; strong scaling).  The inputs cycle
    through a pool of 4 distinct generated layers (6.8 GB per rank, beyond
    L2); outputs go to one buffer per matrix shape.  Each format's launches
    are one CUDA-graph replay timed with CUDA events, max over ranks; value =
    algorithmic bytes (read 2 B/weight, write the packed data and scales) /
    time.  Sampled rows are checked bit-exact against the oracle."""
    import ctypes

    import torch
    import torch.distributed as dist

    from openquant_b200 import _native as nat
    from openquant_b200.sharding import assign_layers

    lib = nat.load()
    mine = assign_layers(layers, world, rank)
    pool = [_bulk_layer(dev, layer) for layer in mine[:min(BULK_POOL, layers)]]
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = {}
    for _, n, k in BULK_SHAPES:
        if (n, k) not in outs:
            outs[(n, k)] = (torch.empty(n * k, dtype=torch.uint8, device=dev),
                            torch.empty(n * (k // 32), dtype=torch.float32, device=dev))
    stream = torch.cuda.Stream(device=dev)
    results = {}
    launches = 0
    for name, g in BULK_FORMATS:
        def launch(layer_ids, h):
            for i, _ in enumerate(layer_ids):
                for (_, n, k), w in zip(BULK_SHAPES, pool[i % len(pool)]):
                    q, sc = outs[(n, k)]
                    if g:
                        st = lib.oq_quant_int4_group(ctypes.c_void_p(w.data_ptr()), nat.OQ_BF16, n, k, g,
                                                     ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                                     ctypes.c_void_p(flag.data_ptr()), h)
                    else:
                        st = lib.oq_quant_int8_rowwise(ctypes.c_void_p(w.data_ptr()), nat.OQ_BF16, n, k,
                                                       ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()), h)
                    if st != 0:
                        raise RuntimeError(nat.last_error())

        with torch.cuda.stream(stream):
            launch(mine[:1], ctypes.c_void_p(stream.cuda_stream))
        stream.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            launch(mine, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        graph.replay()  # warm
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            graph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        del graph
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        launches += len(mine) * len(BULK_SHAPES)
        weights, nbytes = _bulk_bytes(g, layers)
        gbs = nbytes / (ms / 1e3) / 1e9
        results[name] = {"ms": ms, "GB/s": gbs, "Gweights/s": weights / (ms / 1e3) / 1e9,
                         "frac": gbs / world / peaks["hbm_gbs"], "bytes": nbytes}
        # bit-exact spot check: sampled rows of pool layer 0's gate_proj, requantized alone
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oq_oracle as orc

        _, n, k = BULK_SHAPES[4]
        w = pool[0][4]
        q, sc = outs[(n, k)]
        if g:
            st = lib.oq_quant_int4_group(ctypes.c_void_p(w.data_ptr()), nat.OQ_BF16, n, k, g,
                                         ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()),
                                         ctypes.c_void_p(flag.data_ptr()), None)
        else:
            st = lib.oq_quant_int8_rowwise(ctypes.c_void_p(w.data_ptr()), nat.OQ_BF16, n, k,
                                           ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(sc.data_ptr()), None)
        assert st == 0, nat.last_error()
        torch.cuda.synchronize()
        rows = torch.tensor([0, 1, 4097, n - 1], device=dev)
        sample = w[rows].float().cpu().numpy()
        if g:
            d, s_ = orc.quantize_int4_groupwise(sample, g)
            got_d = q[: n * k // 2].view(n, k // 2)[rows].cpu().numpy().reshape(-1)
            got_s = sc[: n * (k // g)].view(n, k // g)[rows].cpu().numpy()
        else:
            d, s_ = orc.quantize(sample, 8)
            got_d = q.view(n, k)[rows].cpu().numpy().view(np.int8)
            got_s = sc[:n][rows].cpu().numpy().reshape(-1, 1)
        assert np.array_equal(got_d.reshape(-1), d.reshape(-1)), name
        assert np.array_equal(got_s.reshape(-1).view(np.uint32), s_.reshape(-1).view(np.uint32)), name
    assert int(flag.item()) == 0
    head = results["int4_g128"]
    weights, _ = _bulk_bytes(128, layers)
    entry = {
        "metric": "bulk quantization GB/s, Llama-3-70B stack (80 layers x 7 matrices, bf16), INT4 g=128",
        "workload": "bulk_quant_llama3_70b_bf16",
        "value": head["GB/s"],
        "unit": "GB/s",
        "ms_per_step": head["ms"],
        "weights_per_step": weights,
        "scaling": "strong",
        "n_gpus": world,
        "formats": results,
        "roofline": {
            "bound": "hbm",
            "achieved": head["GB/s"] / world,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": head["frac"],
            "algorithmic_bytes_per_weight": "2 (bf16 read) + 0.5 (packed) + 4/g (scales); INT8: 2 + 1 + 4/K",
        },
        "config": {"layers": layers, "pool": f"{len(pool)} distinct generated layers cycled ({len(pool) * 1.71:.1f} GB > L2)",
                   "parallelism": f"layers round-robin over {world} GPU(s)",
                   "data": "N(0,0.02) + 0.1% at +-0.2, per-layer seed, generated on the GPU"},
        "gpu_launches": launches,
        "check": "sampled rows of gate_proj bit-exact vs the oracle, every format",
    }
    if rank == 0 and world == 1:
        wps, threads = cpu_bulk_sample()
        per_w = head["bytes"] / weights
        entry["cpu_baseline"] = {"value": wps * per_w / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                                 "sample": f"2048x8192 bf16-valued rows, INT4 g=128 (NumPy restatement of "
                                           f"quantize_int4_groupwise, {threads} threads over row blocks): "
                                           f"{wps / 1e6:.0f} M weights/s"}
    del pool, outs
    torch.cuda.empty_cache()
    return entry


SHARD_K, SHARD_N = 8192, 28672  # Llama-3-70B MLP gate/up projection


def _device_timed(stream, body, steps, host_us_per_step=0.0):
    """ms per step of `body()` (enqueues one step on `stream`) over `steps`
    steps, timed with CUDA events on `stream`.  A device-side sleep is
    enqueued ahead of the start event so that the host has queued the steps
    before the GPU reaches them: the events then bracket device work only."""
    import torch

    cycles = int(2e6 + 2e3 * host_us_per_step * steps)  # ~1 ms + the host's enqueue time at ~2 GHz
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        torch.cuda._sleep(cycles)
        start.record(stream)
        body()
        end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end) / steps


def upload_graph(graph, stream):
    """Uploads an instantiated CUDA graph's work to the device
    (cuGraphUpload) on `stream`, so that its first replay -- inside a timed
    region -- does not carry the upload."""
    import ctypes

    cuda = ctypes.CDLL("libcuda.so.1")
    rc = cuda.cuGraphUpload(ctypes.c_void_p(graph.raw_cuda_graph_exec()), ctypes.c_void_p(stream.cuda_stream))
    if rc != 0:
        raise RuntimeError(f"cuGraphUpload failed ({rc})")


def _max_over_ranks(v, dev, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return v
    t = torch.tensor([v], device=dev, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def measure_sharded(dev, world, rank, peaks, prefill_ms=(2048, 8192), decode_ms=(1, 16)):
    """The N-column-sharded Llama-3-70B gate/up layer (K = 8192, N = 28672,
    INT4 g = 128) over the ranks, each owning N/P contiguous weight rows:

    * p2p  -- the fused path: each rank's kernels store their (M, N/P) slice
              straight into every rank's (M, N) output over NVLink, then a
              bounded flag barrier (ShardedInt4Linear mode "p2p"), fp32 output
              (the reference's) and bf16 output;
    * nccl -- the local slice, then an NCCL all-gather and a relayout copy.

    Prefill at M = 2048 and 8192 (bf16 x) in TFLOP/s of the whole layer,
    decode at M = 1 and 16 (fp16 x) in µs per call.  Each case is timed with
    CUDA events over back-to-back steps (p2p: one CUDA graph of the steps),
    max over ranks, and compared with the same full layer on one GPU
    (`efficiency_vs_1gpu` = t_1gpu / (P * t_P)).  Every rank checks sampled
    columns spanning all shards against the oracle's exactly-rounded weights
    (rel-L2 <= 1e-3 and max-abs <= 2e-2); the bf16 output must equal the fp32
    output rounded once."""
    import torch
    import torch.distributed as dist

    from oq_oracle import dequantize_int4_groupwise as deq, round_to_dtype
    from openquant.triton_int4 import int4_linear
    from openquant_b200.groupwise import Groupwise4, quantize_int4_groupwise
    from openquant_b200.sharding import ShardedInt4Linear, shard_bounds, shard_groupwise

    k, n, g = SHARD_K, SHARD_N, 128
    gen = torch.Generator(device=dev).manual_seed(500)  # the same layer on every rank
    w = torch.randn(n, k, generator=gen, device=dev).mul_(0.02).to(torch.bfloat16)
    q = quantize_int4_groupwise(w, g)
    del w
    sh = shard_groupwise(q, world, rank)
    local = Groupwise4(sh.data.clone(), sh.scales.clone(), sh.shape, g)
    cols = torch.arange(0, n, 1021, device=dev)
    wcols = deq(q.data.view(n, k // 2)[cols].cpu().numpy().reshape(-1), q.scales[cols].cpu().numpy(),
                (len(cols), k), g)
    wround = {torch.bfloat16: torch.from_numpy(round_to_dtype(wcols, "bf16")).to(dev).double(),
              torch.float16: torch.from_numpy(round_to_dtype(wcols, "f16")).to(dev).double()}
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    layers = {mode: ShardedInt4Linear(local, n, mode=mode) for mode in ("p2p", "nccl")}
    a, b = shard_bounds(n, world, rank)
    cases, checks, launches, rel_worst, abs_worst = {}, {}, 0, 0.0, 0.0

    def check(y, x, tag):
        nonlocal rel_worst, abs_worst
        ref = x.double() @ wround[x.dtype].T
        err = y[:, cols].double() - ref
        rel = (err.norm() / ref.norm()).item()
        mab = err.abs().max().item()
        assert rel <= 1e-3 and mab <= 2e-2, (tag, rel, mab)
        rel_worst, abs_worst = max(rel_worst, rel), max(abs_worst, mab)

    def one_gpu_ms(x, steps):
        y1 = torch.empty(x.shape[0], n, device=dev)
        call = lambda: int4_linear(x, q.data, q.scales, n, g, out=y1)  # noqa: E731
        with torch.cuda.stream(stream):
            for _ in range(2):
                call()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(steps):
                    call()
            upload_graph(graph, stream)
        torch.cuda.synchronize()
        ms = _device_timed(stream, graph.replay, steps)
        del graph
        check(y1, x, "1gpu")
        return _max_over_ranks(ms, dev, world)

    def p2p_ms(x, steps, out_dtype):
        lin = layers["p2p"]
        with torch.cuda.stream(stream):
            for _ in range(4):
                y = lin(x, out_dtype=out_dtype)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for _ in range(steps):  # an even count: the two output buffers alternate across replays
                    y = lin(x, out_dtype=out_dtype)
            upload_graph(graph, stream)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        ms = _device_timed(stream, graph.replay, steps)
        del graph
        return _max_over_ranks(ms, dev, world), y

    def nccl_ms(x, steps):
        lin = layers["nccl"]
        with torch.cuda.stream(stream):
            for _ in range(2):
                y = lin(x)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        last = {}

        def body():
            for _ in range(steps):
                last["y"] = lin(x)

        ms = _device_timed(stream, body, steps, host_us_per_step=200.0)
        y = last.pop("y")
        slice_ = torch.empty(x.shape[0], -(-n // world), device=dev)
        flat = torch.empty(world * x.shape[0], slice_.shape[1], device=dev)
        with torch.cuda.stream(stream):
            dist.all_gather_into_tensor(flat, slice_)
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()

        def gather():
            for _ in range(steps):
                dist.all_gather_into_tensor(flat, slice_)

        g_ms = _device_timed(stream, gather, steps, host_us_per_step=100.0)
        return _max_over_ranks(ms, dev, world), _max_over_ranks(g_ms, dev, world), y

    for m in prefill_ms + decode_ms:
        prefill = m >= 64
        xdt = torch.bfloat16 if prefill else torch.float16
        x = torch.randn(m, k, generator=torch.Generator(device=dev).manual_seed(600 + m), device=dev).to(xdt)
        steps = (10 if m <= 2048 else 4) if prefill else 200
        flops = 2.0 * m * n * k
        t1 = one_gpu_ms(x, steps)
        launches += steps + 2
        kind = "prefill" if prefill else "decode"

        def entry(ms):
            e = {"ms": ms, "us": ms * 1e3, "efficiency_vs_1gpu": t1 / (world * ms), "one_gpu_ms": t1}
            if prefill:
                e["tflops"] = flops / (ms / 1e3) / 1e12
                e["per_gpu_frac_of_peak"] = e["tflops"] / world / peaks["bf16_tflops"]
            return e

        ms, y = p2p_ms(x, steps, torch.float32)
        check(y, x, f"p2p m{m}")
        y32 = y[:, cols].clone()
        cases[f"{kind}_m{m}_p2p_f32"] = entry(ms)
        launches += 2 * (steps + 4)
        if prefill:
            ms, yb = p2p_ms(x, steps, torch.bfloat16)
            assert torch.equal(yb[:, cols], y32.bfloat16()), f"bf16 output m{m}"
            cases[f"{kind}_m{m}_p2p_bf16"] = entry(ms)
            launches += 2 * (steps + 4)
        if m in (2048, 1, 16):
            ms, g_ms, y = nccl_ms(x, min(steps, 50))
            check(y, x, f"nccl m{m}")
            e = entry(ms)
            e["allgather_ms"] = g_ms
            cases[f"{kind}_m{m}_nccl_f32"] = e
            launches += min(steps, 50) + 2
        del x, y
    for lin in layers.values():
        lin.close()
    del layers
    torch.cuda.empty_cache()
    head = cases.get("prefill_m2048_p2p_f32")
    return {
        "metric": "N-column-sharded INT4 linear layer (Llama-3-70B gate/up, 8192->28672, g=128): whole-layer "
                  "TFLOP/s at M=2048, fused p2p output",
        "workload": f"int4_linear_sharded{world}_k8192_n28672_g128",
        "value": head["tflops"] if head else None,
        "unit": "TFLOP/s",
        "scaling": "strong",
        "n_gpus": world,
        "shard_rows": [a, b],
        "by_case": cases,
        "modes": {"p2p": "kernels store each output element into every GPU's y over NVLink, then a bounded "
                         "flag barrier (oq_int4_linear_peers + oq_peer_barrier)",
                  "nccl": "local slice, NCCL all_gather_into_tensor, relayout copy"},
        "output_bytes_per_gpu_per_call": {"m2048_f32": 2048 * n * 4 * (world - 1) // world},
        "gpu_launches": launches,
        "check": "every case: sampled columns over all shards vs the oracle's exactly-rounded weights "
                 "(rel-L2 <= 1e-3, max-abs <= 2e-2); bf16 output == fp32 output rounded once",
        "check_rel_l2": rel_worst,
        "check_max_abs": abs_worst,
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)

    from openquant_b200 import _native as nat
    from openquant_b200 import build
    from openquant_b200.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear

    build.build()
    lib = nat.load()
    nat.require_device()

    gen = torch.Generator(device=dev).manual_seed(1000 + rank)
    packs, scs, ys = [], [], []
    for _ in range(COPIES):
        w = torch.randn(N, K, generator=gen, device=dev).mul_(0.02).half()
        q = quantize_int4_groupwise(w, G)
        packs.append(q.data)
        scs.append(q.scales)
        ys.append(torch.empty(M, N, device=dev))
        del w
    x = torch.randn(M, K, generator=gen, device=dev).half()
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device=dev)
    import ctypes

    args_c = [
        (ctypes.c_void_p(x.data_ptr()), nat.OQ_F16, ctypes.c_void_p(packs[i].data_ptr()),
         ctypes.c_void_p(scs[i].data_ptr()), ctypes.c_void_p(ys[i].data_ptr()), M, N, K, G, 0,
         nat.CONFIG_STATIC_WEIGHTS)
        for i in range(COPIES)
    ]

    def launch_many(count, h, first=0):
        for i in range(first, first + count):
            st = lib.oq_int4_linear(*args_c[i % COPIES], h)
            if st != 0:
                raise RuntimeError(nat.last_error())

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    clocks = ClockSampler(uuid)

    def make_graph(first, count):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            launch_many(count, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), first=first)
        upload_graph(g, stream)
        return g

    # Warm-up, exactly W launches: the first eagerly and synchronized -- the
    # kernel's first-launch set-up happens there, before any capture -- the
    # rest right before the timed launches, behind the device-side sleep
    # (up to 64 as plain launches, more as a graph), so that the timed
    # launches follow warm-up launches on the GPU.
    eager = min(args.warmup, 1)
    with torch.cuda.stream(stream):
        launch_many(eager, ctypes.c_void_p(stream.cuda_stream))
    stream.synchronize()
    chunk = 1024
    rest_w = args.warmup - eager
    if rest_w + args.steps <= ONE_GRAPH_MAX:
        graphs = {"warm": make_graph(eager, rest_w) if rest_w > 64 else None,
                  "timed": make_graph(args.warmup, args.steps)}

        def warm():
            if graphs["warm"] is not None:
                graphs["warm"].replay()
            elif rest_w:
                launch_many(rest_w, ctypes.c_void_p(stream.cuda_stream), first=eager)

        def timed():
            graphs["timed"].replay()
    else:
        graphs = {c: make_graph(0, c) for c in {chunk, args.steps % chunk, rest_w % chunk} if c}

        def replay(count):
            """`count` launches: whole chunk graphs, then one graph of the rest."""
            for _ in range(count // chunk):
                graphs[chunk].replay()
            if count % chunk:
                graphs[count % chunk].replay()

        def warm():
            replay(rest_w)

        def timed():
            replay(args.steps)

    torch.cuda.synchronize()
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        # A device-side sleep first: the host submits the warm-up and timed
        # graphs while the GPU sleeps, so the GPU runs the W warm-up launches
        # and then the K timed ones back to back, and the events bracket the
        # timed launches themselves, not the host's submission latency.
        torch.cuda._sleep(int(2e6))
        warm()
        start.record(stream)
        timed()
        end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())

    # correctness spot check of the benchmarked kernel against torch.
    from openquant_b200.groupwise import Groupwise4, dequantize_int4_groupwise

    wref = dequantize_int4_groupwise(Groupwise4(packs[0], scs[0], (N, K), G)).half().double()
    yref = x.double() @ wref.T
    y0 = int4_linear(x, packs[0], scs[0], N, G)
    rel = ((y0.double() - yref).norm() / yref.norm()).item()
    mab = (y0.double() - yref).abs().max().item()
    assert rel <= 1e-3 and mab <= 2e-2, (rel, mab)

    # e2e through the public API with host buffers: Int4Linear.forward_host,
    # x read from and y written to page-locked host memory by the kernel
    # itself (oq_int4_linear_host), one launch and one synchronization a step.
    e2e_steps = E2E_STEPS
    x_host = x.cpu().pin_memory()
    y_hosts = [torch.empty(M, N).pin_memory() for _ in range(2)]
    from openquant.triton_int4 import Int4Linear

    layers = [Int4Linear(packs[i], scs[i], N, G, static_weights=True) for i in range(COPIES)]
    for i in range(min(50, e2e_steps)):
        layers[i % COPIES].forward_host(x_host, out=y_hosts[i & 1])
    y_e2e = layers[0].forward_host(x_host, out=y_hosts[0])
    assert torch.equal(y_e2e, y0.cpu()), "forward_host differs from the device-buffer call"
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for i in range(e2e_steps):
        layers[i % COPIES].forward_host(x_host, out=y_hosts[i & 1])
    e2e_s = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([e2e_s], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    peaks, src = read_peaks()
    step_s = ms / 1e3 / args.steps
    achieved = ALG_BYTES / step_s / 1e9
    value = world * args.steps * ALG_BYTES / (ms / 1e3) / 1e9
    traffic = read_traffic("gemv_m1_k4096_n4096_g128")
    line = {
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic",
        "config": headline_config(world),
        "roofline": {
            "bound": "hbm",
            "achieved": achieved,
            "peak": peaks["hbm_gbs"],
            "unit": "GB/s",
            "frac": achieved / peaks["hbm_gbs"],
            "traffic": traffic,
            "peak_source": src,
            "algorithmic_bytes_per_launch": ALG_BYTES,
        },
        "e2e": {
            "value": world * e2e_steps * ALG_BYTES / e2e_s / 1e9,
            "unit": UNIT,
            "h2d_bytes_per_step": M * K * 2,
            "d2h_bytes_per_step": M * N * 4,
            "steps": e2e_steps,
            "how": "openquant.triton_int4.Int4Linear.forward_host per step (the layer validated once; same kernel "
                   "and result as int4_linear): the kernel reads x from and writes y to page-locked host memory "
                   "(oq_int4_linear_host), then the stream is synchronized; wall clock over all steps",
        },
        "gpu_launches": args.steps,
        "clocks": clk,
        "check_rel_l2": rel,
        "check_max_abs": mab,
    }
    sys.path.insert(0, os.path.join(ROOT, "oracle"))  # the checks below compare against the oracle
    if not args.no_gemm:
        if world == 1:
            line["also"] = [measure_gemm(dev, peaks), measure_w8a8(dev, peaks)]
        else:
            line["also"] = [measure_sharded(dev, world, rank, peaks)]
    if world == 1 and not args.no_layers:
        line.setdefault("also", []).append(measure_decode_layers(dev, peaks))
        if not args.no_gemm:
            line["also"].append(measure_prefill_set(dev, peaks))
        line["also"].append(measure_cpu_path_1024(dev, peaks))
        line["also"].append(measure_gemv_fp16_scales(dev, peaks))
    if not args.no_bulk:
        line.setdefault("also", []).append(measure_bulk_quant(dev, world, rank, peaks, layers=args.bulk_layers))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    del graphs
    line["summary"] = summarize(line)  # last key: the compact figures of every line
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200000)
    ap.add_argument("--warmup", type=int, default=20000)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gemm", action="store_true", help="skip the M=2048 prefill GEMM measurement")
    ap.add_argument("--no-bulk", action="store_true", help="skip the bulk-quantization (70B stack) measurement")
    ap.add_argument("--no-layers", action="store_true", help="skip the Llama-2-7B decode layer-set measurement")
    ap.add_argument("--bulk-layers", type=int, default=BULK_LAYERS,
                    help="layers of the bulk-quantization stack (default 80; fewer for profiling)")
    args = ap.parse_args(argv)
    if args.steps < 1 or args.warmup < 0:
        ap.error("steps must be >= 1 and warmup >= 0")
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
