"""Seeded input recipes for the golden vectors.

Both tests/golden/make_golden.py (which runs the reference package to record
its outputs) and the tests (which rebuild the same inputs to check the oracle
and the CUDA kernels) import this module, so every input is regenerated
bit-for-bit from its recipe rather than stored.
"""
from __future__ import annotations

import numpy as np


def bf16_exact(a):
    """Truncate fp32 values to the nearest bf16 (ties to even) so that the
    same numbers can be fed to the kernels as fp32, fp16-free bf16 or fp32."""
    a = np.asarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    u = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return u.astype(np.uint32).view(np.float32)


def _ties_rowwise(qmax):
    # Rows whose max is qmax, so the scale is exactly 1.0 and every other
    # entry is a quotient that sits exactly on a rounding tie.
    vals = np.array([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, 5.5, 6.5, -6.5], np.float32)
    row0 = np.concatenate([[qmax], vals]).astype(np.float32)
    row1 = np.concatenate([[-qmax], vals * 2.0]).astype(np.float32)  # scale 1, even/odd ints
    row2 = np.concatenate([[qmax * 0.25], vals * 0.25]).astype(np.float32)  # scale 0.25, ties
    return np.stack([row0, row1, row2])


def _edge_rowwise():
    return np.array(
        [
            [np.nan, 1.0, 2.0, -3.0],
            [np.inf, 1.0, -1.0, 0.0],
            [1e-45, -1e-45, 0.0, 0.0],
            [3e-39, 1e-39, 0.0, 0.0],
            [0.0, 0.0, 0.0, 0.0],
            [-np.inf, -np.inf, 5.0, np.nan],
        ],
        dtype=np.float32,
    )


def rowwise_cases():
    """name -> fp32 weight matrix for quantize(bits=4/8)."""
    cases = {}
    r = np.random.default_rng(100)
    cases["std_5x7"] = r.standard_normal((5, 7)).astype(np.float32)
    r = np.random.default_rng(100)
    cases["std_1x1"] = r.standard_normal((1, 1)).astype(np.float32)
    r = np.random.default_rng(100)
    cases["std_3x1"] = r.standard_normal((3, 1)).astype(np.float32)
    r = np.random.default_rng(42)
    cases["n1_128x256"] = r.normal(size=(128, 256)).astype(np.float32)
    cases["ones_17x19"] = np.ones((17, 19), np.float32)
    cases["zero_row_3x3"] = np.array([[0, 0, 0], [1, -1, 0.5], [0, -0.5, 1]], np.float32)
    r = np.random.default_rng(3)
    cases["n002_33x65"] = r.normal(0, 0.02, (33, 65)).astype(np.float32)
    r = np.random.default_rng(4)
    cases["n02_9x31_bf16"] = bf16_exact(r.normal(0, 0.2, (9, 31)))
    r = np.random.default_rng(5)
    cases["n002_64x1000"] = r.normal(0, 0.02, (64, 1000)).astype(np.float32)
    cases["ties_int8"] = _ties_rowwise(127.0)
    cases["ties_int4"] = _ties_rowwise(7.0)
    cases["edge_nonfinite"] = _edge_rowwise()
    return cases


def group_cases():
    """name -> (fp32 weights, group_size) for quantize_int4_groupwise."""
    cases = {}
    for shape in [(3, 67), (5, 32), (1, 1)]:
        for g in (16, 32):
            r = np.random.default_rng(7)
            cases[f"n1_{shape[0]}x{shape[1]}_g{g}"] = (r.normal(size=shape).astype(np.float32), g)
    cases["zeros_2x35_g32"] = (np.zeros((2, 35), np.float32), 32)
    r = np.random.default_rng(11)
    cases["n1_4x8_g2"] = (r.normal(size=(4, 8)).astype(np.float32), 2)
    r = np.random.default_rng(12)
    cases["n1_6x40_g6"] = (r.normal(size=(6, 40)).astype(np.float32), 6)
    r = np.random.default_rng(13)
    cases["n002_7x130_g128"] = (r.normal(0, 0.02, (7, 130)).astype(np.float32), 128)
    r = np.random.default_rng(14)
    cases["n002_9x300_g64"] = (r.normal(0, 0.02, (9, 300)).astype(np.float32), 64)
    r = np.random.default_rng(15)
    cases["n002_16x512_g8_bf16"] = (bf16_exact(r.normal(0, 0.02, (16, 512))), 8)
    r = np.random.default_rng(16)
    cases["n002_32x4096_g128_bf16"] = (bf16_exact(r.normal(0, 0.02, (32, 4096))), 128)
    r = np.random.default_rng(17)
    cases["n002_24x96_g256"] = (r.normal(0, 0.02, (24, 96)).astype(np.float32), 256)
    r = np.random.default_rng(18)
    cases["n002_5x100_g12"] = (r.normal(0, 0.02, (5, 100)).astype(np.float32), 12)
    t = _ties_rowwise(7.0)  # 3 x 13, g=13 is odd: use g=14 (one padded group)
    cases["ties_3x13_g14"] = (t, 14)
    return cases


def outlier_weights(rng, shape, sigma=0.02, frac=0.001):
    """N(0, sigma) with `frac` of the entries set to +-10 sigma, the
    bulk-quantization weight model (70B stack, 0.1 % outliers)."""
    w = rng.normal(0, sigma, shape).astype(np.float32)
    count = max(1, int(round(frac * w.size)))
    idx = rng.choice(w.size, size=count, replace=False)
    w.reshape(-1)[idx] = np.where(rng.random(count) < 0.5, -10 * sigma, 10 * sigma).astype(np.float32)
    return w


def hashed_cases():
    """Full-size cases whose outputs are stored only as SHA-256 digests.

    name -> (kind, recipe); recipe() returns the fp32 input, `kind` is
    ("rowwise", bits) or ("group", g)."""

    def cfg1():
        # 1024x1024 ~ N(0, 0.02), seed 0: the CPU-path workload.
        return np.random.default_rng(0).normal(0, 0.02, (1024, 1024)).astype(np.float32)

    def gemv4096():
        # 4096x4096 ~ N(0, 0.02), the decode GEMV weight (weight seed 1).
        return np.random.default_rng(1).normal(0, 0.02, (4096, 4096)).astype(np.float32)

    def outl():
        return bf16_exact(outlier_weights(np.random.default_rng(2), (1024, 8192)))

    return {
        "cfg1_int8": (("rowwise", 8), cfg1),
        "cfg1_int4": (("rowwise", 4), cfg1),
        "cfg1_g32": (("group", 32), cfg1),
        "gemv4096_g128": (("group", 128), gemv4096),
        "outlier_1024x8192_int8": (("rowwise", 8), outl),
        "outlier_1024x8192_g128": (("group", 128), outl),
        "outlier_1024x8192_g32": (("group", 32), outl),
    }
