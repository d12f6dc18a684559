"""Record golden vectors by running the reference package itself.

Usage (in a container where the reference source tree is mounted):

    python tests/golden/make_golden.py <path of the reference source tree>

It imports the reference's openquant package from the given tree, runs its
NumPy quantizers / dequantizers and its torch decode helpers (on CPU
tensors) on the seeded inputs of tests/golden/cases.py, and writes
tests/golden/golden.npz (packed bytes and scales of every small case, and
their fp32 outputs up to 8192 elements) and tests/golden/golden_hashes.json
(SHA-256 of the larger fp32 outputs and of the full-size cases' bytes).
Nothing at test or bench time reads the reference tree.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import warnings

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref_root):
    sys.path.insert(0, HERE)
    sys.path.insert(0, ref_root)
    import torch  # noqa: F401  (the reference helpers are torch functions)
    from openquant.quantization import quantize, dequantize
    from openquant.groupwise import quantize_int4_groupwise, dequantize_int4_groupwise
    from openquant.gpu_benchmark import decode_gpu
    from openquant.group_benchmark import restore_groupwise_torch
    import openquant

    assert os.path.abspath(openquant.__file__).startswith(os.path.abspath(ref_root)), openquant.__file__
    import cases

    out = {}
    digests = {}

    def put(key, arr):
        # Small arrays are stored whole; large float outputs as digests.
        arr = np.ascontiguousarray(arr)
        if arr.dtype == np.float32 and arr.size > 8192:
            digests[key] = sha(arr)
        else:
            out[key] = arr

    warnings.simplefilter("ignore")
    for name, w in cases.rowwise_cases().items():
        for bits in (8, 4):
            q = quantize(w, bits)
            key = f"row{bits}/{name}"
            put(key + "/data", q.data)
            put(key + "/scales", q.scales)
            put(key + "/dequant", dequantize(q))
            dec = decode_gpu(torch.from_numpy(q.data), torch.from_numpy(q.scales), bits, w.shape)
            put(key + "/decode_gpu", dec.numpy())
    for name, (w, g) in cases.group_cases().items():
        q = quantize_int4_groupwise(w, g)
        key = f"group/{name}"
        put(key + "/data", q.data)
        put(key + "/scales", q.scales)
        put(key + "/dequant", dequantize_int4_groupwise(q))
        rest = restore_groupwise_torch(torch.from_numpy(q.data), torch.from_numpy(q.scales), w.shape, g)
        put(key + "/restore_torch", rest.contiguous().numpy())
    np.savez_compressed(os.path.join(HERE, "golden.npz"), **out)

    hashes = {}
    for name, ((kind, param), recipe) in cases.hashed_cases().items():
        w = recipe()
        if kind == "rowwise":
            q = quantize(w, param)
        else:
            q = quantize_int4_groupwise(w, param)
        hashes[name] = {
            "kind": kind,
            "param": param,
            "shape": list(w.shape),
            "data_sha256": sha(q.data),
            "data_nbytes": int(q.data.nbytes),
            "scales_sha256": sha(q.scales),
            "scales_shape": list(q.scales.shape),
        }
    with open(os.path.join(HERE, "golden_hashes.json"), "w") as f:
        json.dump({"cases": hashes, "arrays": digests}, f, indent=1, sort_keys=True)
        f.write("\n")
    print(f"wrote {len(out)} arrays, {len(digests)} digests, {len(hashes)} hashed cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference source tree>")
    main(sys.argv[1])
