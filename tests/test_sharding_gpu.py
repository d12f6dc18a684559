"""The N-column-sharded fused linear on 2 GPUs over NCCL vs one GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, queue):
    from datetime import timedelta

    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60), device_id=dev)
        from openquant_b200.groupwise import quantize_int4_groupwise
        from openquant_b200.sharding import ShardedInt4Linear, quantize_layers, shard_groupwise
        from openquant_b200.triton_int4 import int4_linear

        n, k, g = 1000, 2048, 128
        gen = torch.Generator(device=dev).manual_seed(3)
        w = torch.randn(n, k, device=dev, generator=gen).mul_(0.02).half()
        x = torch.randn(300, k, device=dev, generator=gen).to(torch.bfloat16)
        q = quantize_int4_groupwise(w, g)
        full = int4_linear(x, q.data, q.scales, n, g)
        y = ShardedInt4Linear(shard_groupwise(q, world, rank), n)(x)
        err = (y - full).abs().max().item()
        xs = x[:4].half()
        ys = ShardedInt4Linear(shard_groupwise(q, world, rank), n)(xs)
        errs = (ys - int4_linear(xs, q.data, q.scales, n, g)).abs().max().item()
        owned = quantize_layers(lambda i: torch.randn(64, 256, device=dev), 5, group_size=64)
        dist.destroy_process_group()
        queue.put((rank, err, errs, sorted(owned)))
    except Exception as exc:
        queue.put((rank, repr(exc), None, None))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_linear_two_gpus():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(queue.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    for rank, err, errs, owned in res:
        assert isinstance(err, float), err
        assert err < 1e-3 and errs < 1e-3, (rank, err, errs)
        assert owned == [i for i in range(5) if i % 2 == rank]
