"""Builds the openquant_b200 CUDA library in-tree.

    python -m openquant_b200.build [--force] [--verbose]

Every .cu file under openquant_b200/csrc is compiled for sm_100a (nvcc
-gencode arch=compute_100a,code=sm_100a, no fast-math: the quantizers rely on
IEEE division and denormals) and linked into
openquant_b200/_lib/libopenquant_b200.so, which the Python package loads
with ctypes.  Objects go to openquant_b200/_build/.  A file is recompiled
when it or any header is newer than its object.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libopenquant_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def cflags():
    return ARCH + [
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC,-O3,-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-I" + os.path.join(ROOT, "include"),
        "-I" + CSRC,
    ]


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(force=False, verbose=False, ptxas_verbose=False):
    """Compile and link the library; returns its path."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    header_time = _newest(headers + [os.path.abspath(__file__)])

    def compile_one(src):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        if not force and os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), header_time):
            return obj, None
        cmd = [nvcc, "-c", src, "-o", obj] + cflags()
        if ptxas_verbose:
            cmd += ["-Xptxas", "-v"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
        return obj, (res.stdout + res.stderr) if (verbose or ptxas_verbose) else None

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as pool:
        results = list(pool.map(compile_one, sources))
    for _, log in results:
        if log:
            sys.stderr.write(log)
    objs = [o for o, _ in results]
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, "-shared", "-o", tmp] + objs + ARCH + ["-lcuda"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true", help="print register / shared-memory usage")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas_verbose))


if __name__ == "__main__":
    main()
