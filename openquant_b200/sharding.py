"""Multi-GPU sharding of the quantize-and-multiply path.

Two decompositions, one process per GPU (torch.distributed, NCCL over NVLink):

* N-column sharding of a fused INT4 linear layer: rank r holds a contiguous block of
  weight rows (output features) -- rows of the packed Groupwise4 data (each row is
  KP/2 contiguous bytes) and of the (N, G) scales -- and computes its slice of
  y = x . W^T; the slices reach every GPU either through the kernels' own
  stores into peer-mapped outputs over NVLink (fused) or through an NCCL
  all-gather.  x is replicated.
* layer partitioning of bulk quantization: whole matrices are assigned to ranks
  round-robin; no collective on the data path.

The reference (openquant 0.5.0) is single-GPU; this module adds the sharding the
build's large layers and bulk stack are distributed with.  The per-rank compute
function is a parameter so the collective logic can be exercised on CPU ranks.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import tile_table
from .groupwise import Groupwise4, padded_cols

__all__ = [
    "shard_bounds",
    "shard_groupwise",
    "ShardedInt4Linear",
    "PeerBuffers",
    "assign_layers",
    "quantize_layers",
]


def shard_bounds(n_total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced row range [start, end) of `rank` among `world`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(int(n_total), world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_groupwise(q: Groupwise4, world: int, rank: int) -> Groupwise4:
    """The rows of a groupwise-quantized matrix owned by `rank` (views, no copy
    when `q` lives on the target device)."""
    rows, cols = (int(v) for v in q.shape)
    kp = padded_cols(cols, q.group_size)
    start, end = shard_bounds(rows, world, rank)
    data = q.data.reshape(rows, kp // 2)[start:end].reshape(-1)
    scales = q.scales[start:end]
    return Groupwise4(data=data, scales=scales, shape=(end - start, cols), group_size=q.group_size)


def _default_linear(x, packed, scales, n_local, group_size):
    from .triton_int4 import int4_linear

    return int4_linear(x, packed, scales, n_local, group_size)


class _DeviceArray:
    """A device pointer presented to torch through __cuda_array_interface__."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


_TYPESTR = {torch.float32: ("<f4", None), torch.float16: ("<f2", None), torch.bfloat16: ("<i2", torch.bfloat16)}


class PeerBuffers:
    """Device buffers of the given sizes on every rank's GPU, each mapped into
    every rank of `group` (CUDA IPC over NVLink: plain peer mappings).

    Collective: every rank constructs it with the same sizes.  ptrs[i][r] is
    buffer i of rank r as an address this process can store to; ptrs[i][rank]
    is this GPU's own buffer.  close() (collective too) unmaps the peers'
    buffers, then frees this rank's once no rank maps it any more.
    """

    def __init__(self, sizes, group=None):
        from . import _native as nat

        self._nat = nat
        self.lib = nat.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.local, handles = [], []
        try:
            for nbytes in sizes:
                p = ctypes.c_void_p()
                nat.check(self.lib.oq_peer_alloc(int(nbytes), ctypes.byref(p)))
                self.local.append(p.value)
                h = (ctypes.c_uint8 * nat.PEER_HANDLE_BYTES)()
                nat.check(self.lib.oq_peer_export(ctypes.c_void_p(p.value), h))
                handles.append(bytes(h))
        except Exception:
            for p in self.local:
                self.lib.oq_peer_free(ctypes.c_void_p(p))
            raise
        everyone = [None] * self.world
        dist.all_gather_object(everyone, handles, group=group)
        self.imported = []
        self.ptrs = []
        for i in range(len(sizes)):
            row = []
            for r in range(self.world):
                if r == self.rank:
                    row.append(self.local[i])
                    continue
                p = ctypes.c_void_p()
                h = (ctypes.c_uint8 * nat.PEER_HANDLE_BYTES).from_buffer_copy(everyone[r][i])
                nat.check(self.lib.oq_peer_import(h, ctypes.byref(p)))
                self.imported.append(p.value)
                row.append(p.value)
            self.ptrs.append(row)

    def view(self, i, shape, dtype):
        """Buffer i of this GPU as a torch tensor (no copy; valid until close())."""
        typestr, as_dtype = _TYPESTR[dtype]
        t = torch.as_tensor(_DeviceArray(self.local[i], shape, typestr), device=torch.cuda.current_device())
        return t.view(as_dtype) if as_dtype is not None else t

    def close(self):
        if self.local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.imported:
            self.lib.oq_peer_close(ctypes.c_void_p(p))
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.local:
            self.lib.oq_peer_free(ctypes.c_void_p(p))
        self.local = self.imported = self.ptrs = None


@dataclass
class ShardedInt4Linear:
    """y = x . W^T with W's rows sharded across the ranks of `group`.

    `local` is this rank's shard (shard_groupwise), `n_total` the full number
    of output features.  Every rank calls it with the same x (replicated) and
    gets the full (M, N) y.  Two ways to assemble y:

    * mode "p2p" (the default on CUDA): one fused step -- this GPU's kernels
      (oq_int4_linear_peers: the decode GEMV or the tcgen05 GEMM, whichever
      int4_linear would run for the local shape) store every element of the
      local slice straight into the y buffer of every GPU over NVLink while
      the tiles are computed, then a flag barrier on the stream
      (oq_peer_barrier, bounded wait) orders the stream's next work after all
      peers' stores into this GPU's y.  No gather or relayout pass.  The
      output buffers are peer-mapped and allocated collectively on the first
      call of each (M, out dtype) -- every rank must make the same calls --
      and two of them alternate, so a returned y stays valid for work
      enqueued on the stream before the next call of the layer; copy it to
      keep it longer.  close() releases them (collective).
    * mode "nccl": the local slice by `linear` (default int4_linear), then an
      NCCL all-gather of the (M, N/P) slices (padded to ceil(N/P) columns)
      and one strided copy into y.  This also runs on CPU ranks (gloo) with a
      CPU `linear`, which the tests use for the collective logic.
    """

    local: Groupwise4
    n_total: int
    group: object = None
    linear: object = None
    mode: str = None

    def __post_init__(self):
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        self.start, self.end = shard_bounds(self.n_total, self.world, self.rank)
        if self.end - self.start != int(self.local.shape[0]):
            raise ValueError("local shard has the wrong number of rows for this rank")
        self.n_pad = -(-self.n_total // self.world)
        if self.mode is None:
            self.mode = "p2p" if self.linear is None and self.local.data.is_cuda and self.world > 1 else "nccl"
        if self.mode not in ("p2p", "nccl"):
            raise ValueError("mode must be 'p2p' or 'nccl'")
        if self.mode == "p2p" and (self.linear is not None or not self.local.data.is_cuda):
            raise ValueError("mode 'p2p' runs the library's CUDA kernels on CUDA tensors")
        if self.world > 8 and self.mode == "p2p":
            raise ValueError("mode 'p2p' takes at most 8 GPUs")
        if self.linear is None:
            self.linear = _default_linear
        self._flags = None
        self._outs = {}
        self._calls = 0

    # ---------------------------------------------------------- nccl --
    def _call_nccl(self, x):
        n_local = self.end - self.start
        m = int(x.shape[0])
        y_local = self.linear(x, self.local.data, self.local.scales, n_local, self.local.group_size)
        if self.world == 1:
            return y_local
        send = y_local
        if n_local < self.n_pad:  # uneven split: pad the slice
            send = torch.zeros((m, self.n_pad), dtype=y_local.dtype, device=y_local.device)
            send[:, :n_local] = y_local
        flat = torch.empty((self.world * m, self.n_pad), dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(flat, send.contiguous(), group=self.group)
        gathered = flat.view(self.world, m, self.n_pad)
        if self.n_total == self.world * self.n_pad:  # even split: one strided copy into (M, N)
            return gathered.permute(1, 0, 2).reshape(m, self.n_total)
        y = torch.empty((m, self.n_total), dtype=y_local.dtype, device=y_local.device)
        for r in range(self.world):
            a, b = shard_bounds(self.n_total, self.world, r)
            y[:, a:b] = gathered[r, :, : b - a]
        return y

    # ----------------------------------------------------------- p2p --
    def _buffers(self, m, dtype):
        from . import _native as nat

        key = (m, dtype)
        if key not in self._outs:
            if self._flags is None:
                self._flags = PeerBuffers([4 * nat.PEER_FLAG_WORDS], self.group)
            esize = torch.empty((), dtype=dtype).element_size()
            bufs = PeerBuffers([m * self.n_total * esize] * 2, self.group)
            views = [bufs.view(i, (m, self.n_total), dtype) for i in range(2)]
            self._outs[key] = (bufs, views)
        return self._outs[key]

    def _call_p2p(self, x, out_dtype, bias):
        from . import _native as nat
        from .triton_int4 import _YCODES, _stream_handle

        if x.ndim != 2 or x.dtype not in (torch.float16, torch.bfloat16) or not x.is_cuda or not x.is_contiguous():
            raise ValueError("x must be a contiguous 2-D fp16 or bf16 CUDA tensor")
        if out_dtype not in _YCODES:
            raise ValueError("out_dtype must be torch.float32, torch.float16 or torch.bfloat16")
        m, k = (int(v) for v in x.shape)
        if int(self.local.shape[1]) != k:
            raise ValueError("x has the wrong number of columns for this layer")
        n_local = self.end - self.start
        if bias is not None and (bias.dtype != torch.float32 or bias.numel() != n_local or not bias.is_cuda):
            raise ValueError("bias must be this shard's float32 CUDA tensor of N/P elements")
        bufs, views = self._buffers(m, out_dtype)
        slot = self._calls & 1
        self._calls += 1
        world, rank = self.world, self.rank
        order = [(rank + j) % world for j in range(world)]  # this GPU first, then its peers in rank order
        ys = (ctypes.c_void_p * world)(*[bufs.ptrs[slot][r] for r in order])
        flags = (ctypes.c_void_p * world)(*self._flags.ptrs[0])
        g = int(self.local.group_size)
        sel, split = tile_table.lookup(m, n_local, k, g)
        lib = nat.load()
        dev = x.get_device()
        stream = _stream_handle(dev)
        code = nat.OQ_F16 if x.dtype == torch.float16 else nat.OQ_BF16

        def run(sel, split):
            ws_bytes = lib.oq_int4_linear_workspace_bytes(m, n_local, k, g, sel, split) if m > 16 else 0
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device) if ws_bytes else None
            return lib.oq_int4_linear_peers(x.data_ptr(), code, self.local.data.data_ptr(),
                                            self.local.scales.data_ptr(), ys, world, _YCODES[out_dtype],
                                            bias.data_ptr() if bias is not None else None, self.n_total,
                                            self.start, m, n_local, k, g, sel, split,
                                            ws.data_ptr() if ws is not None else None, ws_bytes, stream)

        status = run(sel, split)
        if status == nat.OQ_ERR_INVALID and (sel, split) != (0, 0):
            status = run(0, 0)  # a tuned launch shape of the M bucket that rejects this M
        nat.check(status)
        nat.check(lib.oq_peer_barrier(flags, world, rank, 0, stream))
        return views[slot]

    def __call__(self, x, out_dtype=torch.float32, bias=None):
        if self.mode == "p2p":
            return self._call_p2p(x, out_dtype, bias)
        if out_dtype != torch.float32 or bias is not None:
            raise ValueError("mode 'nccl' writes fp32 without bias")
        return self._call_nccl(x)

    def close(self):
        """Releases the peer-mapped buffers of mode 'p2p' (collective)."""
        for bufs, _ in self._outs.values():
            bufs.close()
        self._outs = {}
        if self._flags is not None:
            self._flags.close()
            self._flags = None


def assign_layers(num_layers: int, world: int, rank: int) -> list[int]:
    """Round-robin layer ownership for bulk quantization."""
    return [i for i in range(int(num_layers)) if i % world == rank]


def quantize_layers(make_weight, num_layers: int, group_size=None, bits=None, world=None, rank=None):
    """Quantize this rank's share of a layer stack.

    `make_weight(i)` returns layer i's weight (a tensor on this rank's GPU);
    with `group_size` the groupwise INT4 quantizer is used, with `bits` (4 or
    8) the per-row one.  Returns {layer index: quantized result} for the
    layers this rank owns.  No collective: layers are independent.
    """
    from .groupwise import quantize_int4_groupwise
    from .quantization import quantize

    if (group_size is None) == (bits is None):
        raise ValueError("pass exactly one of group_size (groupwise INT4) or bits (per-row)")
    if world is None:
        world = dist.get_world_size() if dist.is_initialized() else 1
    if rank is None:
        rank = dist.get_rank() if dist.is_initialized() else 0
    out = {}
    for i in assign_layers(num_layers, world, rank):
        w = make_weight(i)
        out[i] = quantize_int4_groupwise(w, group_size) if group_size is not None else quantize(w, bits)
    return out
