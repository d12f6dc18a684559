"""N-column sharding and layer partitioning, checked with gloo ranks on CPU.

The per-rank compute is the oracle (the collective logic is what is under
test); the CUDA path of the same class is covered by test_sharding_gpu.py.
"""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oq_oracle as orc
from openquant_b200.groupwise import Groupwise4
from openquant_b200.sharding import ShardedInt4Linear, assign_layers, shard_bounds, shard_groupwise


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def oracle_linear(x, packed, scales, n_local, group_size):
    xn = x.numpy()
    y = orc.int4_linear(xn, np.asarray(packed), np.asarray(scales), n_local, group_size, x_dtype="f16")
    return torch.from_numpy(y)


def make_layer(n, k, g, seed=0):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    data, scales = orc.quantize_int4_groupwise(w, g)
    return Groupwise4(data=data, scales=scales, shape=(n, k), group_size=g)


def _worker(rank, world, port, n, k, g, m, queue):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        q = make_layer(n, k, g)
        x = torch.from_numpy(np.random.default_rng(5).normal(size=(m, k)).astype(np.float32))
        lin = ShardedInt4Linear(shard_groupwise(q, world, rank), n, linear=oracle_linear)
        y = lin(x).numpy()
        ref = orc.int4_linear(x.numpy(), q.data, q.scales, n, g, x_dtype="f16")
        queue.put((rank, float(np.abs(y - ref).max()), y.shape))
        dist.destroy_process_group()
    except Exception as exc:  # report to the parent
        queue.put((rank, repr(exc), None))


@pytest.mark.parametrize("world,n", [(2, 37), (2, 64), (3, 10)])
def test_sharded_linear_matches_full_product(world, n):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, 96, 32, 3, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, err, shape in results:
        assert shape == (3, n), (rank, err)
        assert err == 0.0, (rank, err)


def test_shard_bounds_cover_rows():
    for n in (1, 7, 16, 28672):
        for world in (1, 2, 3, 8):
            spans = [shard_bounds(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_shard_groupwise_rows_and_layer_assignment():
    q = make_layer(10, 70, 32)
    kp = 96
    parts = [shard_groupwise(q, 3, r) for r in range(3)]
    np.testing.assert_array_equal(np.concatenate([p.data for p in parts]), q.data)
    np.testing.assert_array_equal(np.concatenate([p.scales for p in parts]), q.scales)
    assert [p.shape for p in parts] == [(4, 70), (3, 70), (3, 70)]
    assert parts[0].data.size == 4 * kp // 2
    owned = [assign_layers(80, 8, r) for r in range(8)]
    assert sorted(sum(owned, [])) == list(range(80))
    assert all(len(o) == 10 for o in owned)


def _dropout_worker(rank, world, port, queue):
    from datetime import timedelta

    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=3))
        if rank == 1:
            queue.put((rank, "left"))  # leaves between steps: never enters the collective
            time.sleep(8)
            return
        q = make_layer(16, 64, 32)
        lin = ShardedInt4Linear(shard_groupwise(q, world, rank), 16, linear=oracle_linear)
        t0 = time.time()
        try:
            lin(torch.zeros(2, 64))
            queue.put((rank, "no error"))
        except Exception as exc:
            queue.put((rank, f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"))
    except Exception as exc:
        queue.put((rank, repr(exc)))


def test_peer_that_leaves_makes_the_collective_fail_not_hang():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert results[1] == "left"
    assert results[0].startswith("error after"), results[0]
