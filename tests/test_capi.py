"""The C-ABI library builds, loads without a GPU and exports every entry
point declared in include/*.h; the Python API validates its arguments
before touching a device and never falls back to the CPU.  CPU only."""
import glob
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT

HEADERS = glob.glob(os.path.join(ROOT, "include", "*.h"))


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(oq_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from openquant_b200 import build, _native

    build.build()
    return _native.load()


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "oq_int4_linear" in names and "oq_quant_int4_group" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol(lib):
    import ctypes

    raw = ctypes.CDLL(lib._name)
    for name in declared_symbols():
        assert hasattr(raw, name), f"{name} declared in include/ but not exported"


def test_binding_covers_header(lib):
    from openquant_b200 import _native

    assert set(_native.SIGNATURES) == set(declared_symbols())


def test_version_and_error_without_gpu(lib):
    assert lib.oq_version().decode().startswith("openquant_b200")
    assert lib.oq_last_error() is not None
    if not torch.cuda.is_available():
        assert lib.oq_device_count() <= 0


def test_argument_errors_come_from_the_library(lib):
    # Argument checks run before any CUDA call, so they work without a GPU.
    from openquant_b200 import _native

    st = lib.oq_int4_linear(None, 7, None, None, None, 1, 1, 1, 32, 0, 0, None)
    assert st == _native.OQ_ERR_INVALID
    assert "FP16" in _native.last_error()
    st = lib.oq_quant_int4_group(None, 0, 4, 4, 3, None, None, None, None)
    assert st == _native.OQ_ERR_INVALID and "even" in _native.last_error()
    st = lib.oq_quant_int8_rowwise(None, 0, 0, 4, None, None, None)
    assert st == _native.OQ_ERR_INVALID


def test_python_validation_errors_without_gpu():
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.quantization import quantize
    from openquant.triton_int4 import int4_linear

    with pytest.raises(ValueError):
        quantize(np.ones((2, 2)), bits=3)
    with pytest.raises(ValueError):
        quantize(np.ones(10), bits=8)
    for g in (0, 1, 3):
        with pytest.raises(ValueError):
            quantize_int4_groupwise(np.ones((2, 8)), g)
    with pytest.raises(ValueError):
        quantize_int4_groupwise(np.ones(8))
    with pytest.raises(ValueError):
        quantize_int4_groupwise(np.zeros((3, 0)))
    x = torch.zeros(2, 8, dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        int4_linear(x, torch.zeros(8, dtype=torch.uint8), torch.zeros(2, 1), 2, 8)
    with pytest.raises(ValueError, match="FP16"):
        int4_linear(x.float(), torch.zeros(8, dtype=torch.uint8), torch.zeros(2, 1), 2, 8)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    from openquant.gpu_benchmark import decode_gpu
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.quantization import quantize

    with pytest.raises(RuntimeError):
        quantize(np.ones((2, 2), np.float32), 8)
    with pytest.raises(RuntimeError):
        quantize_int4_groupwise(np.ones((2, 8), np.float32), 8)
    with pytest.raises(RuntimeError):
        decode_gpu(torch.zeros(4, dtype=torch.int8), torch.ones(2, 1), 8, (2, 2))
