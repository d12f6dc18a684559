"""Kernel / split-K table for int4_linear.

`openquant tune` (openquant_b200.autotune) times every kernel variant on a
set of shapes on the B200 and writes the winners to tile_table.json next to
this file; lookup() reads it once.  Without a table entry the C library's
own shape rule picks the kernel (kernel code 0, "auto").
"""
from __future__ import annotations

import json
import os

TABLE_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tile_table.json")
_table = None


def m_bucket(m):
    """Batch-size bucket: 1, 2, 4, ..., 64, then 128+ buckets by powers of 2."""
    b = 1
    while b < m:
        b *= 2
    return b


def load_table(path=TABLE_PATH):
    global _table
    if _table is None:
        try:
            with open(path) as f:
                data = json.load(f)
            _table = {tuple(e["key"]): (int(e["kernel"]), int(e.get("split_k", 0))) for e in data.get("entries", [])}
        except (OSError, ValueError, KeyError):
            _table = {}
    return _table


def reset():
    global _table
    _table = None


def lookup(m, n, k, g):
    """(kernel code, split_k) for this shape; (0, 0) = library default."""
    return load_table().get((m_bucket(m), n, k, g), (0, 0))
