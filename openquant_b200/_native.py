"""ctypes binding of the openquant_b200 C ABI (include/openquant_b200.h).

The library is built in-tree by openquant_b200.build.  There is no CPU
fallback: when the library is missing or no sm_100 device is present, the
entry points raise RuntimeError instead of computing anything on the host.
"""
from __future__ import annotations

import ctypes
import os
import threading

import numpy as np

from .build import LIB

OQ_OK, OQ_ERR_INVALID, OQ_ERR_CUDA, OQ_ERR_UNSUPPORTED = 0, 1, 2, 3
OQ_F32, OQ_F16, OQ_BF16, OQ_F64 = 0, 1, 2, 3
KERNELS = {"auto": 0, "gemv": 1, "simt": 2, "tcgen05": 3}
CONFIG_EXACT_ROUNDING = 16
CONFIG_STATIC_WEIGHTS = 32
CONFIG_SILU_GATE = 64

# name -> (restype, argtypes), exactly the declarations of the header.
_P, _I64, _I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
SIGNATURES = {
    "oq_version": (ctypes.c_char_p, []),
    "oq_last_error": (ctypes.c_char_p, []),
    "oq_device_count": (_I32, []),
    "oq_take_device_error": (_I32, [_P]),
    "oq_quant_int8_rowwise": (_I32, [_P, _I32, _I64, _I64, _P, _P, _P]),
    "oq_quant_int4_rowwise": (_I32, [_P, _I32, _I64, _I64, _P, _P, _P]),
    "oq_quant_int4_group": (_I32, [_P, _I32, _I64, _I64, _I32, _P, _P, _P, _P]),
    "oq_dequant_int8_rowwise": (_I32, [_P, _P, _I64, _I64, _P, _P]),
    "oq_dequant_int4_rowwise": (_I32, [_P, _P, _I64, _I64, _P, _P]),
    "oq_dequant_int4_group": (_I32, [_P, _P, _I64, _I64, _I32, _P, _P]),
    "oq_int4_linear": (_I32, [_P, _I32, _P, _P, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P]),
    "oq_int8_gemm": (_I32, [_P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    "oq_int4_linear_ex": (_I32, [_P, _I32, _P, _P, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P]),
    "oq_int8_linear_noalloc": (_I32, [_P, _I32, _P, _P, _P, _I64, _I64, _I64, _P]),
    "oq_int4_linear_peers": (_I32, [_P, _I32, _P, _P, _P, _I32, _I32, _P, _I64, _I64, _I64, _I64, _I64, _I32, _I32,
                                    _I32, _P, ctypes.c_size_t, _P]),
    "oq_int4_linear_ws": (_I32, [_P, _I32, _P, _P, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P,
                                 ctypes.c_size_t, _P]),
    "oq_int4_linear_workspace_bytes": (_I64, [_I64, _I64, _I64, _I32, _I32, _I32]),
    "oq_int4_linear_f16s": (_I32, [_P, _I32, _P, _P, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32, _P]),
    "oq_int4_linear_host": (_I32, [_P, _I32, _P, _P, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P, _P]),
    "oq_int4_linear_host_plan": (_I32, [_P, _I32, _P, _P, _P, _I32, _P, _I64, _I64, _I64, _I32, _I32, _I32, _P,
                                        _P]),
    "oq_int4_linear_host_run": (_I32, [_P, _P]),
    "oq_int4_linear_host_plan_free": (_I32, [_P]),
    "oq_peer_alloc": (_I32, [ctypes.c_size_t, _P]),
    "oq_peer_free": (_I32, [_P]),
    "oq_peer_export": (_I32, [_P, _P]),
    "oq_peer_import": (_I32, [_P, _P]),
    "oq_peer_close": (_I32, [_P]),
    "oq_peer_barrier": (_I32, [_P, _I32, _I32, _I64, _P]),
}
PEER_HANDLE_BYTES = 64
PEER_FLAG_WORDS = 16

_lock = threading.Lock()
_lib = None


def library_path():
    return LIB


def load():
    """Load (once) and return the ctypes library; RuntimeError if absent."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB):
                raise RuntimeError(
                    f"openquant_b200 CUDA library not found at {LIB}; build it with "
                    "`python -m openquant_b200.build` (there is no CPU fallback)"
                )
            lib = ctypes.CDLL(LIB)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error():
    return load().oq_last_error().decode(errors="replace")


def check(status, what=""):
    if status == OQ_OK:
        return
    msg = last_error() or what
    if status == OQ_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


_device_ok = None


def require_device():
    """RuntimeError unless torch sees CUDA and the library sees an sm_100 GPU."""
    global _device_ok
    import torch

    if _device_ok:
        return
    if not torch.cuda.is_available():
        raise RuntimeError("openquant_b200 runs its kernels on a CUDA device (B200, sm_100a); none is available")
    n = load().oq_device_count()
    if n < 1:
        raise RuntimeError("openquant_b200 needs a compute-capability 10.x GPU (B200); none was found")
    _device_ok = True


def torch_dtype_code(dtype):
    import torch

    codes = {torch.float32: OQ_F32, torch.float16: OQ_F16, torch.bfloat16: OQ_BF16, torch.float64: OQ_F64}
    return codes.get(dtype)


def numpy_dtype_code(dtype):
    codes = {np.dtype(np.float32): OQ_F32, np.dtype(np.float16): OQ_F16, np.dtype(np.float64): OQ_F64}
    return codes.get(np.dtype(dtype))


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream_of(device):
    import torch

    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr_of_stream(stream):
    return ctypes.c_void_p(stream.cuda_stream)
