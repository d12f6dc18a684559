"""int4_linear: fused groupwise-INT4 dequant + matmul on the B200.

Drop-in for openquant/triton_int4.py:78-138.  The module keeps the
reference's name so `from openquant.triton_int4 import int4_linear` keeps
working, but it contains no Triton: the call goes through the C ABI
(oq_int4_linear) to hand-written sm_100a kernels -- a tensor-core GEMV for
the decode side (M <= 64), the tcgen05/TMEM GEMM for the prefill side, and a
CUDA-core kernel for shapes neither covers.
"""
from __future__ import annotations

import torch

from . import _native as nat
from . import tile_table

__all__ = ["int4_linear", "Int4Linear"]

_YCODES = {torch.float32: nat.OQ_F32, torch.float16: nat.OQ_F16, torch.bfloat16: nat.OQ_BF16}
_PLANS = 8  # captured host-buffer calls an Int4Linear keeps (forward_host)
# The current stream's handle of a device without building a Stream object
# (a decode step calls int4_linear once per layer: host overhead counts).
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_handle(dev):
    if _raw_stream is not None:
        return _raw_stream(dev)
    return torch.cuda.current_stream(dev).cuda_stream


def int4_linear(x, packed, scales, out_features, group_size, *, block_m=64, block_n=64, block_k=64, num_warps=4,
                kernel=None, out=None, exact_rounding=False, static_weights=False, bias=None, out_dtype=None,
                silu_gate=False, fp16_scales=False):
    """y = x @ W^T in fp32, W[n, k] = round_x(int4(n, k) * scales[n, k // g]).

    Arguments and errors follow triton_int4.py:78-118 (ValueError for each
    failed precondition), except that x may also be bf16.  The weight is
    rounded to x's dtype after the fp32 multiply, as the reference kernel
    does (triton_int4.py:62-65), and products accumulate in fp32.

    block_m / block_n / block_k / num_warps are the reference's Triton tile
    arguments; they are accepted (autotune-style callers pass them) and have
    no effect on the result.  Kernel choice comes from the tuned tile table
    (openquant_b200/tile_table.json) or `kernel` ("gemv", "simt",
    "tcgen05"); `out` may supply a preallocated fp32 (M, N) tensor.
    The launch is asynchronous on the current CUDA stream of x's device.

    With fp16 x, M <= 16 and group_size % 128 == 0 the decode GEMV
    multiplies x by the exact integer nibbles and applies each fp32 group
    scale to the group's fp32 partial sum (closer to x.(q*s) than the
    reference, and within the parity tolerance of it).  exact_rounding=True
    instead rounds every weight to fp16 as the reference kernel does, bit
    for bit; bf16 x and larger M always do.

    bias (fp32 [N] on x's device) is added to every output row and out_dtype
    (torch.float32 by default, or torch.float16 / torch.bfloat16) is the type
    y is written in -- both fused into the kernel's epilogue: the bias is
    added in fp32 and the sum rounded once.  With out= the output's dtype is
    used.

    silu_gate=True fuses the gate/up pair of an MLP: `packed` and `scales`
    hold the [gate; up] stack (2 * out_features rows, gate first) and y is
    silu(x . Wg^T) * (x . Wu^T) with silu(g) = g / (1 + exp(-g)), computed in
    one pass (no bias): the decode GEMV for M <= 16, else the tcgen05 GEMM,
    whose tiles pair each feature's gate and up rows so its epilogue writes
    silu(gate) * up directly.

    static_weights=True declares that `packed` and `scales` were written
    before any kernel still in flight on the stream (quantized at load time
    and synchronized): the decode GEMV then streams them while the previous
    kernel drains instead of after it.  Results are unchanged.

    fp16_scales=True takes `scales` as fp16 (N, G) -- one fp16 scale per
    group, half the scale bytes -- instead of the reference's fp32 (which
    stays the default and the only format without the flag): the weights are
    int4 * (float)scale, run on the decode GEMV's scale-after mode (fp16 x,
    M <= 16, group_size a multiple of 128), which applies each scale to its
    group's sum.
    """
    if x.ndim != 2 or x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("Input must be a 2D FP16 tensor")
    if not x.is_cuda or not packed.is_cuda or not scales.is_cuda:
        raise ValueError("All tensors must be on CUDA")
    if not x.is_contiguous():
        raise ValueError("Input must be contiguous")
    if packed.dtype != torch.uint8:
        raise ValueError("Packed weights must be uint8")
    if scales.dtype != (torch.float16 if fp16_scales else torch.float32):
        raise ValueError("Scales must be float16 (fp16_scales=True)" if fp16_scales else "Scales must be float32")
    if group_size < 2 or group_size % 2:
        raise ValueError("Group size must be even and >= 2")
    m, k = (int(v) for v in x.shape)
    n = int(out_features)
    g = int(group_size)
    kp = ((k + g - 1) // g) * g
    groups = kp // g
    if m < 1 or n < 1 or k < 1:
        raise ValueError("Matrix dimensions must be positive")
    rows = 2 * n if silu_gate else n  # weight rows: the [gate; up] stack with silu_gate
    if tuple(scales.shape) != (rows, groups):
        raise ValueError("Incorrect scales shape")
    if packed.numel() != rows * kp // 2:
        raise ValueError("Incorrect packed weight count")
    if silu_gate and bias is not None:
        raise ValueError("silu_gate takes no bias")
    if not packed.is_contiguous() or not scales.is_contiguous():
        raise ValueError("Weights and scales must be contiguous")
    dev = x.get_device()
    if packed.get_device() != dev or scales.get_device() != dev:
        raise ValueError("All tensors must use the same GPU")
    for v in (block_m, block_n, block_k, num_warps):
        if int(v) < 1:
            raise ValueError("Tile arguments must be positive")

    ycodes = _YCODES
    if out is None:
        odt = torch.float32 if out_dtype is None else out_dtype
        if odt not in ycodes:
            raise ValueError("out_dtype must be torch.float32, torch.float16 or torch.bfloat16")
        out = torch.empty((m, n), device=x.device, dtype=odt)
    elif (out.shape != (m, n) or out.dtype not in ycodes or out.get_device() != dev or not out.is_contiguous()
          or (out_dtype is not None and out.dtype != out_dtype)):
        raise ValueError("out must be a contiguous float32, float16 or bfloat16 (M, N) tensor on x's device")
    if bias is not None:
        if (not isinstance(bias, torch.Tensor) or bias.dtype != torch.float32 or bias.numel() != n
                or bias.get_device() != dev or not bias.is_contiguous()):
            raise ValueError("bias must be a contiguous float32 tensor of N elements on x's device")

    nat.require_device()
    if fp16_scales:
        if silu_gate or kernel not in (None, "gemv") or exact_rounding:
            raise ValueError("fp16_scales runs the decode GEMV's scale-after mode (no silu_gate, exact_rounding or "
                             "kernel choice)")
        lib = nat.load()

        def launch_f16s():
            nat.check(lib.oq_int4_linear_f16s(x.data_ptr(), nat.OQ_F16 if x.dtype == torch.float16 else nat.OQ_BF16,
                                              packed.data_ptr(), scales.data_ptr(), out.data_ptr(), ycodes[out.dtype],
                                              bias.data_ptr() if bias is not None else None, m, n, k, g,
                                              nat.CONFIG_STATIC_WEIGHTS if static_weights else 0, _stream_handle(dev)))

        if torch.cuda.current_device() == dev:
            launch_f16s()
        else:
            with torch.cuda.device(dev):
                launch_f16s()
        return out
    if silu_gate:
        if kernel not in (None, "gemv", "tcgen05"):
            raise ValueError("silu_gate runs on the GEMV (M <= 16) or the tcgen05 GEMM")
        sel, split = nat.KERNELS[kernel or "auto"], nat.CONFIG_SILU_GATE
    elif kernel is None:
        sel, split = tile_table.lookup(m, n, k, g)
    else:
        if kernel not in nat.KERNELS:
            raise ValueError(f"unknown kernel {kernel!r}")
        sel, split = nat.KERNELS[kernel], 0
    if exact_rounding:
        split |= nat.CONFIG_EXACT_ROUNDING
    if static_weights:
        split |= nat.CONFIG_STATIC_WEIGHTS
    code = nat.OQ_F16 if x.dtype == torch.float16 else nat.OQ_BF16
    from_table = kernel is None and not silu_gate and (sel, split & 15) != (0, 0)

    lib = nat.load()
    ptrs = (x.data_ptr(), packed.data_ptr(), scales.data_ptr(), out.data_ptr())
    plain = bias is None and out.dtype == torch.float32 and not silu_gate

    def run(sel, split):
        stream = _stream_handle(dev)
        ws_bytes = lib.oq_int4_linear_workspace_bytes(m, n, k, g, sel, split) if m > 16 else 0
        if ws_bytes > 0:  # the prefill GEMM's even split of uneven tile counts (stream-K)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
            return lib.oq_int4_linear_ws(ptrs[0], code, ptrs[1], ptrs[2], ptrs[3], ycodes[out.dtype],
                                         bias.data_ptr() if bias is not None else None, m, n, k, g, sel, split,
                                         ws.data_ptr(), ws_bytes, stream)
        if plain:
            return lib.oq_int4_linear(ptrs[0], code, ptrs[1], ptrs[2], ptrs[3], m, n, k, g, sel, split, stream)
        return lib.oq_int4_linear_ex(ptrs[0], code, ptrs[1], ptrs[2], ptrs[3], ycodes[out.dtype],
                                     bias.data_ptr() if bias is not None else None, m, n, k, g, sel, split, stream)

    def launch():
        status = run(sel, split)
        if status == nat.OQ_ERR_INVALID and from_table:
            # A tuned launch shape is chosen per batch-size bucket; a smaller or
            # larger M in the bucket can fall outside its shared-memory plan.
            status = run(0, split & ~15)
        nat.check(status)

    # The library works on the current device: switch only when x lives elsewhere.
    if torch.cuda.current_device() == dev:
        launch()
    else:
        with torch.cuda.device(dev):
            launch()
    return out


class Int4Linear:
    """int4_linear for one fixed quantized weight, validated once.

    A decode step calls the same layers over and over; this object checks
    the weight-side arguments (packed, scales, out_features, group_size, bias,
    out_dtype -- the preconditions of int4_linear, triton_int4.py:90-118 of
    the reference) when it is made, and each call then checks only x (2-D
    fp16 or bf16, contiguous, on the weights' GPU, K columns that pad to the
    weights' KP) and launches the library's kernel directly -- the same
    kernel and launch shape int4_linear chooses, so the same result bit for
    bit.  `out`, when given, must be a contiguous (M, N) tensor of out_dtype
    on that GPU; the call returns it (a new tensor otherwise).
    """

    def __init__(self, packed, scales, out_features, group_size, *, bias=None, out_dtype=torch.float32,
                 exact_rounding=False, static_weights=False, kernel=None):
        if not packed.is_cuda or not scales.is_cuda:
            raise ValueError("All tensors must be on CUDA")
        if packed.dtype != torch.uint8:
            raise ValueError("Packed weights must be uint8")
        if scales.dtype != torch.float32:
            raise ValueError("Scales must be float32")
        g = int(group_size)
        if g < 2 or g % 2:
            raise ValueError("Group size must be even and >= 2")
        n = int(out_features)
        if n < 1 or scales.ndim != 2 or int(scales.shape[0]) != n or int(scales.shape[1]) < 1:
            raise ValueError("Incorrect scales shape")
        kp = int(scales.shape[1]) * g
        if packed.numel() != n * kp // 2:
            raise ValueError("Incorrect packed weight count")
        if not packed.is_contiguous() or not scales.is_contiguous():
            raise ValueError("Weights and scales must be contiguous")
        dev = packed.get_device()
        if scales.get_device() != dev:
            raise ValueError("All tensors must use the same GPU")
        if out_dtype not in _YCODES:
            raise ValueError("out_dtype must be torch.float32, torch.float16 or torch.bfloat16")
        if bias is not None and (not isinstance(bias, torch.Tensor) or bias.dtype != torch.float32
                                 or bias.numel() != n or bias.get_device() != dev or not bias.is_contiguous()):
            raise ValueError("bias must be a contiguous float32 tensor of N elements on the weights' GPU")
        if kernel is not None and kernel not in nat.KERNELS:
            raise ValueError(f"unknown kernel {kernel!r}")
        nat.require_device()
        self.packed, self.scales, self.bias = packed, scales, bias
        self.out_features, self.group_size, self.out_dtype = n, g, out_dtype
        self._kp, self._dev, self._kernel = kp, dev, kernel
        self._flags = (nat.CONFIG_EXACT_ROUNDING if exact_rounding else 0) | (
            nat.CONFIG_STATIC_WEIGHTS if static_weights else 0)
        self._lib = nat.load()
        self._plain = bias is None and out_dtype == torch.float32
        self._ptrs = (packed.data_ptr(), scales.data_ptr(), bias.data_ptr() if bias is not None else None)
        self._ycode = _YCODES[out_dtype]
        self._device = torch.device("cuda", dev)
        self._shapes = {}  # m -> (kernel code, config, from the tuned table)
        self._stages = {}  # (m, k) -> device copy of a host x (forward_host)
        self._plans = {}  # (x ptr, out ptr, m, k, dtype) -> (plan handle, x, out) (forward_host)

    def _choice(self, m, k):
        sel, split = (tile_table.lookup(m, self.out_features, k, self.group_size) if self._kernel is None
                      else (nat.KERNELS[self._kernel], 0))
        from_table = self._kernel is None and (sel, split & 15) != (0, 0)
        cfg = split | self._flags
        ws = self._lib.oq_int4_linear_workspace_bytes(m, self.out_features, k, self.group_size, sel, cfg) if m > 16 \
            else 0
        c = (sel, cfg, from_table, ws)
        self._shapes[(m, k)] = c
        return c

    def __call__(self, x, out=None):
        if x.dtype is torch.float16:
            code = nat.OQ_F16
        elif x.dtype is torch.bfloat16:
            code = nat.OQ_BF16
        else:
            raise ValueError("Input must be a 2D FP16 tensor")
        if x.ndim != 2 or not x.is_cuda or x.get_device() != self._dev or not x.is_contiguous():
            raise ValueError("x must be a contiguous 2-D tensor on the weights' GPU")
        m, k = x.shape
        g = self.group_size
        if m < 1 or (k + g - 1) // g * g != self._kp:
            raise ValueError("x has the wrong number of columns for these weights")
        n = self.out_features
        if out is None:
            out = torch.empty((m, n), device=self._device, dtype=self.out_dtype)
        elif (out.dtype is not self.out_dtype or out.shape != (m, n) or out.get_device() != self._dev
              or not out.is_contiguous()):
            raise ValueError("out must be a contiguous (M, N) tensor of out_dtype on the weights' GPU")
        if torch.cuda.current_device() != self._dev:  # the library launches on the current device
            with torch.cuda.device(self._dev):
                return self(x, out)
        sel, cfg, from_table, ws_bytes = self._shapes.get((m, k)) or self._choice(m, k)
        stream = _stream_handle(self._dev)
        p, s, b = self._ptrs
        if ws_bytes:  # the prefill GEMM's even split (stream-K) needs a workspace
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self._device)
            st = self._lib.oq_int4_linear_ws(x.data_ptr(), code, p, s, out.data_ptr(), self._ycode, b, m, n, k, g,
                                             sel, cfg, ws.data_ptr(), ws_bytes, stream)
            if st == nat.OQ_ERR_INVALID and from_table:
                st = self._lib.oq_int4_linear_ws(x.data_ptr(), code, p, s, out.data_ptr(), self._ycode, b, m, n, k,
                                                 g, 0, cfg & ~15, ws.data_ptr(), ws_bytes, stream)
        elif self._plain:
            st = self._lib.oq_int4_linear(x.data_ptr(), code, p, s, out.data_ptr(), m, n, k, g, sel, cfg, stream)
            if st == nat.OQ_ERR_INVALID and from_table:
                st = self._lib.oq_int4_linear(x.data_ptr(), code, p, s, out.data_ptr(), m, n, k, g, 0, cfg & ~15,
                                              stream)
        else:
            st = self._lib.oq_int4_linear_ex(x.data_ptr(), code, p, s, out.data_ptr(), self._ycode, b, m, n, k, g,
                                             sel, cfg, stream)
            if st == nat.OQ_ERR_INVALID and from_table:
                st = self._lib.oq_int4_linear_ex(x.data_ptr(), code, p, s, out.data_ptr(), self._ycode, b, m, n, k,
                                                 g, 0, cfg & ~15, stream)
        if st:
            nat.check(st)
        return out

    def forward_host(self, x, out=None):
        """The layer on host tensors: x a contiguous (M, K) fp16 / bf16 CPU
        tensor in page-locked memory (``pin_memory()``), the result written
        into `out` -- a page-locked (M, N) CPU tensor of out_dtype, allocated
        when None -- and returned once it is complete.  A small kernel copies
        x over the bus into a device buffer this object keeps per M, while the
        layer kernel's weights stream; the layer kernel writes y straight into
        `out`.  The first call with a given (x, out) pair captures both
        kernels into a CUDA graph (oq_int4_linear_host_plan) that later calls
        with the same tensors replay -- one graph launch and one
        synchronization per decode step; the object keeps those tensors alive
        while it holds their plan (the last _PLANS pairs).  The same kernel
        and result as ``self(x.cuda()).cpu()`` -- bit for bit for decode
        shapes; the prefill GEMM runs without its stream-K split.  The
        weights' GPU must be the current device."""
        # (page-locking of x and out is checked by the library, which refuses
        # pageable memory with OQ_ERR_INVALID -> ValueError)
        if x.dtype is torch.float16:
            code = nat.OQ_F16
        elif x.dtype is torch.bfloat16:
            code = nat.OQ_BF16
        else:
            raise ValueError("Input must be a 2D FP16 tensor")
        if x.ndim != 2 or x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous 2-D CPU tensor in page-locked memory (pin_memory())")
        m, k = x.shape
        g, n = self.group_size, self.out_features
        if m < 1 or (k + g - 1) // g * g != self._kp:
            raise ValueError("x has the wrong number of columns for these weights")
        if out is None:
            out = torch.empty((m, n), dtype=self.out_dtype, pin_memory=True)
        elif out.dtype is not self.out_dtype or out.shape != (m, n) or out.is_cuda or not out.is_contiguous():
            raise ValueError("out must be a contiguous page-locked (M, N) CPU tensor of out_dtype")
        key = (x.data_ptr(), out.data_ptr(), m, k, code)
        entry = self._plans.get(key)
        if entry is None:
            entry = self._make_plan(x, out, code)
        st = self._lib.oq_int4_linear_host_run(entry[0], _stream_handle(self._dev))
        if st:
            nat.check(st)
        return out

    def _make_plan(self, x, out, code):
        import ctypes

        m, k = x.shape
        g, n = self.group_size, self.out_features
        stage = self._stages.get((m, k))
        if stage is None:
            stage = self._stages[(m, k)] = torch.empty((m, k), dtype=torch.float16, device=self._device)
        sel, cfg, from_table, _ = self._shapes.get((m, k)) or self._choice(m, k)
        p, s, b = self._ptrs
        args = (x.data_ptr(), code, p, s, out.data_ptr(), self._ycode, b, m, n, k, g)
        handle = ctypes.c_void_p()
        st = self._lib.oq_int4_linear_host_plan(*args, sel, cfg, stage.data_ptr(), ctypes.byref(handle))
        if st == nat.OQ_ERR_INVALID and from_table:
            st = self._lib.oq_int4_linear_host_plan(*args, 0, cfg & ~15, stage.data_ptr(), ctypes.byref(handle))
        if st:
            nat.check(st)
        if len(self._plans) >= _PLANS:  # drop the oldest plan (dicts keep insertion order)
            old = self._plans.pop(next(iter(self._plans)))
            self._lib.oq_int4_linear_host_plan_free(old[0])
        entry = (handle, x, out)  # the plan reads and writes these tensors' memory
        self._plans[(x.data_ptr(), out.data_ptr(), m, k, code)] = entry
        return entry

    def __del__(self):
        plans = getattr(self, "_plans", None)
        if plans:
            try:
                for handle, _, _ in plans.values():
                    self._lib.oq_int4_linear_host_plan_free(handle)
            except Exception:  # interpreter shutdown: the process's graphs go with it
                pass
            plans.clear()
