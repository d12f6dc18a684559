"""Multi-GPU sharding of the quantize-and-multiply path.

Two decompositions, one process per GPU (torch.distributed, NCCL over NVLink):

* N-column sharding of a fused INT4 linear layer: rank r holds a contiguous block of
  weight rows (output features) -- rows of the packed Groupwise4 data (each row is
  KP/2 contiguous bytes) and of the (N, G) scales -- and computes its slice of
  y = x . W^T; an all-gather of the (M, N/P) fp32 slices assembles y.  x is
  replicated.
* layer partitioning of bulk quantization: whole matrices are assigned to ranks
  round-robin; no collective on the data path.

The reference (openquant 0.5.0) is single-GPU; this module adds the sharding the
build's large layers and bulk stack are distributed with.  The per-rank compute
function is a parameter so the collective logic can be exercised on CPU ranks.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from .groupwise import Groupwise4, padded_cols

__all__ = [
    "shard_bounds",
    "shard_groupwise",
    "ShardedInt4Linear",
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


@dataclass
class ShardedInt4Linear:
    """y = x . W^T with W's rows sharded across the ranks of `group`.

    `local` is this rank's shard (shard_groupwise), `n_total` the full number
    of output features.  Calling it computes the local slice with `linear`
    (default: openquant_b200.triton_int4.int4_linear on the local GPU) and
    all-gathers the slices (slices are padded to ceil(N/P) columns so the
    collective moves equal sizes).  Every rank returns the full (M, N) fp32 y.
    """

    local: Groupwise4
    n_total: int
    group: object = None
    linear: object = None

    def __post_init__(self):
        self.world = dist.get_world_size(self.group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(self.group) if dist.is_initialized() else 0
        self.start, self.end = shard_bounds(self.n_total, self.world, self.rank)
        if self.end - self.start != int(self.local.shape[0]):
            raise ValueError("local shard has the wrong number of rows for this rank")
        self.n_pad = -(-self.n_total // self.world)
        if self.linear is None:
            self.linear = _default_linear

    def __call__(self, x):
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
        pieces = [gathered[r, :, : shard_bounds(self.n_total, self.world, r)[1] - shard_bounds(self.n_total, self.world, r)[0]]
                  for r in range(self.world)]
        return torch.cat(pieces, dim=1)


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
