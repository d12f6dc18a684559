"""On-disk packed weights: save Groupwise4 / QuantizedWeights and stream them
back into HBM.

The reference keeps quantized weights only in memory (groupwise.py:5-10,
quantization.py:6-11).  This file format stores them exactly as they are laid
out for the kernels, so loading is one sequential read and a stream of
host-to-device copies, with no re-packing:

    bytes 0..7     magic b"OQB2CKPT"
    bytes 8..15    header length H (little-endian uint64)
    bytes 16..     H bytes of UTF-8 JSON:
                   {"format": "openquant_b200.checkpoint", "version": 1,
                    "entries": {name: {"kind": "groupwise4" | "quantized",
                                       "shape": [rows, cols],
                                       "group_size": g  |  "bits": 4 or 8,
                                       "arrays": {"data": {...}, "scales": {...}}}}}
                   each array: {"dtype", "shape", "offset", "nbytes"}
    payload        every array at a 4096-byte aligned offset, in header order

load(path, device="cuda") allocates every destination tensor first, then
reads the payload in large chunks into two pinned host buffers -- a reader
thread fills one while the copy stream moves the other to the GPU -- so disk
reads and PCIe transfers overlap.  Chunks may straddle arrays.
"""
from __future__ import annotations

import json
import os
import struct
import threading

import numpy as np

from .groupwise import Groupwise4
from .quantization import QuantizedWeights

__all__ = ["save", "load"]

MAGIC = b"OQB2CKPT"
ALIGN = 4096
_DTYPES = {"uint8": np.uint8, "int8": np.int8, "float32": np.float32}


def _host(a):
    try:
        import torch

        if isinstance(a, torch.Tensor):
            return a.detach().cpu().numpy()
    except ImportError:  # pragma: no cover - torch is a dependency of the package
        pass
    return np.asarray(a)


def _entry(obj):
    if isinstance(obj, Groupwise4):
        return {"kind": "groupwise4", "shape": [int(v) for v in obj.shape], "group_size": int(obj.group_size)}
    if isinstance(obj, QuantizedWeights):
        return {"kind": "quantized", "shape": [int(v) for v in obj.shape], "bits": int(obj.bits)}
    raise TypeError(f"cannot save {type(obj).__name__}: expected Groupwise4 or QuantizedWeights")


def save(path, weights: dict):
    """Write `weights` ({name: Groupwise4 | QuantizedWeights}, numpy or torch
    data on any device) to `path`."""
    arrays = []
    entries = {}
    for name, obj in weights.items():
        ent = _entry(obj)
        ent["arrays"] = {}
        for field in ("data", "scales"):
            a = np.ascontiguousarray(_host(getattr(obj, field)))
            if a.dtype.name not in _DTYPES:
                raise TypeError(f"{name}.{field}: unsupported dtype {a.dtype}")
            ent["arrays"][field] = {"dtype": a.dtype.name, "shape": list(a.shape), "nbytes": int(a.nbytes)}
            arrays.append((ent["arrays"][field], a))
        entries[str(name)] = ent
    header = {"format": "openquant_b200.checkpoint", "version": 1, "entries": entries}
    # offsets depend on the header length: fix the header size first with
    # placeholder offsets of the final width, then fill them in
    for meta, _ in arrays:
        meta["offset"] = 0
    for _ in range(3):
        blob = json.dumps(header, separators=(",", ":")).encode()
        off = -(-(16 + len(blob)) // ALIGN) * ALIGN
        for meta, a in arrays:
            meta["offset"] = off
            off += -(-a.nbytes // ALIGN) * ALIGN
    blob = json.dumps(header, separators=(",", ":")).encode()
    start = -(-(16 + len(blob)) // ALIGN) * ALIGN
    if arrays and arrays[0][0]["offset"] != start:
        raise RuntimeError("checkpoint header layout did not converge")
    with open(path, "wb") as f:
        f.write(MAGIC + struct.pack("<Q", len(blob)) + blob)
        for meta, a in arrays:
            f.seek(meta["offset"])
            f.write(a.tobytes())
        end = arrays[-1][0]["offset"] + arrays[-1][0]["nbytes"] if arrays else 16 + len(blob)
        f.truncate(end)


def _read_header(f):
    head = f.read(16)
    if len(head) != 16 or head[:8] != MAGIC:
        raise ValueError("not an openquant_b200 checkpoint (bad magic)")
    (hlen,) = struct.unpack("<Q", head[8:])
    blob = f.read(hlen)
    if len(blob) != hlen:
        raise ValueError("truncated checkpoint header")
    header = json.loads(blob)
    if header.get("format") != "openquant_b200.checkpoint" or header.get("version") != 1:
        raise ValueError("unsupported checkpoint format or version")
    return header


def _build(entries, arrays):
    out = {}
    for name, ent in entries.items():
        data, scales = arrays[(name, "data")], arrays[(name, "scales")]
        shape = tuple(ent["shape"])
        if ent["kind"] == "groupwise4":
            out[name] = Groupwise4(data=data, scales=scales, shape=shape, group_size=ent["group_size"])
        elif ent["kind"] == "quantized":
            out[name] = QuantizedWeights(data=data, scales=scales, bits=ent["bits"], shape=shape)
        else:
            raise ValueError(f"{name}: unknown entry kind {ent['kind']!r}")
    return out


def load(path, device="cuda", chunk_bytes=64 << 20):
    """Read a checkpoint: {name: Groupwise4 | QuantizedWeights} with numpy
    arrays (device="cpu") or torch tensors on `device` (a CUDA device), the
    latter streamed through two pinned buffers of `chunk_bytes`."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        header = _read_header(f)
    entries = header["entries"]
    metas = [(name, field, ent["arrays"][field]) for name, ent in entries.items() for field in ("data", "scales")]
    for name, field, meta in metas:
        if meta["dtype"] not in _DTYPES:
            raise ValueError(f"{name}.{field}: unsupported dtype {meta['dtype']}")
        if meta["offset"] % ALIGN or meta["offset"] + meta["nbytes"] > size:
            raise ValueError(f"{name}.{field}: array outside the file (truncated checkpoint?)")
        if int(np.prod(meta["shape"], dtype=np.int64)) * np.dtype(_DTYPES[meta["dtype"]]).itemsize != meta["nbytes"]:
            raise ValueError(f"{name}.{field}: shape and size disagree")

    if str(device) == "cpu":
        arrays = {}
        with open(path, "rb") as f:
            for name, field, meta in metas:
                f.seek(meta["offset"])
                raw = f.read(meta["nbytes"])
                arrays[(name, field)] = np.frombuffer(raw, dtype=_DTYPES[meta["dtype"]]).reshape(meta["shape"]).copy()
        return _build(entries, arrays)

    import torch

    from . import _native as nat

    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("device must be 'cpu' or a CUDA device")
    nat.require_device()
    tdt = {"uint8": torch.uint8, "int8": torch.int8, "float32": torch.float32}
    arrays = {(n, fld): torch.empty(m["shape"], dtype=tdt[m["dtype"]], device=dev) for n, fld, m in metas}
    # Byte ranges of the payload: (file offset, nbytes, destination byte view).
    spans = sorted(((m["offset"], m["nbytes"], arrays[(n, fld)].view(-1).view(torch.uint8))
                    for n, fld, m in metas if m["nbytes"]), key=lambda s: s[0])
    if not spans:
        return _build(entries, arrays)
    lo, hi = spans[0][0], spans[-1][0] + spans[-1][1]
    chunk = int(max(ALIGN, min(chunk_bytes, hi - lo)))
    bufs = [torch.empty(chunk, dtype=torch.uint8).pin_memory() for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    stream = torch.cuda.Stream(device=dev)
    filled = [threading.Semaphore(0), threading.Semaphore(0)]
    free = [threading.Semaphore(1), threading.Semaphore(1)]
    n_chunks = -(-(hi - lo) // chunk)
    lengths = [min(chunk, hi - lo - i * chunk) for i in range(n_chunks)]
    error = []

    def reader():
        try:
            with open(path, "rb", buffering=0) as f:
                f.seek(lo)
                for i, ln in enumerate(lengths):
                    b = i & 1
                    free[b].acquire()
                    view = memoryview(bufs[b].numpy())[:ln]
                    got = 0
                    while got < ln:
                        r = f.readinto(view[got:])
                        if not r:
                            raise ValueError("truncated checkpoint payload")
                        got += r
                    filled[b].release()
        except Exception as exc:  # surfaced to the caller below
            error.append(exc)
            for s in filled:
                s.release()

    th = threading.Thread(target=reader, daemon=True)
    th.start()
    si = 0
    with torch.cuda.stream(stream):
        for i, ln in enumerate(lengths):
            b = i & 1
            filled[b].acquire()
            if error:
                break
            c0, c1 = lo + i * chunk, lo + i * chunk + ln
            while si < len(spans) and spans[si][0] + spans[si][1] <= c0:
                si += 1
            j = si
            while j < len(spans) and spans[j][0] < c1:
                off, nb, dst = spans[j]
                a, z = max(off, c0), min(off + nb, c1)
                dst[a - off:z - off].copy_(bufs[b][a - c0:z - c0], non_blocking=True)
                j += 1
            copied[b].record(stream)
            # the reader may refill this buffer once its copies have run
            copied[b].synchronize()
            free[b].release()
    th.join()
    stream.synchronize()
    if error:
        raise error[0]
    return _build(entries, arrays)
