"""The N-column-sharded fused linear layer on the GPU.

One GPU: oq_int4_linear_peers storing one shard's columns into several
output buffers (stand-ins for the peers' buffers) against the plain entry
point and the oracle; the flag barrier with its peer's flag preset and with a
flag that nothing sets (the wait must run out and report it); a peer buffer
exported by this process and written by another one (CUDA IPC).
Two GPUs: the sharded layer in both modes (p2p stores + barrier, and the NCCL
all-gather) against the unsharded layer.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oq_oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    from openquant_b200 import build

    build.build()


def _lib():
    from openquant_b200 import _native as nat

    return nat, nat.load()


def _take_device_error():
    nat, lib = _lib()
    code = ctypes.c_int32(-1)
    nat.check(lib.oq_take_device_error(ctypes.byref(code)))
    return code.value


def _ptrs(ts):
    return (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])


CASES = [  # m, n_total, k, g, kernel, x dtype
    (1, 1000, 2048, 128, "gemv", torch.float16),
    (16, 1000, 2048, 128, "gemv", torch.float16),
    (5, 700, 1024, 64, "gemv", torch.bfloat16),
    (300, 1000, 2048, 128, "tcgen05", torch.bfloat16),
    (77, 500, 512, 32, "tcgen05", torch.float16),
    (9, 300, 200, 8, "simt", torch.float16),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"m{c[0]}_n{c[1]}_k{c[2]}_g{c[3]}_{c[4]}")
@pytest.mark.parametrize("y_dtype", [torch.float32, torch.bfloat16])
def test_peers_entry_writes_every_buffer(case, y_dtype):
    """Three shards, each written by oq_int4_linear_peers into three output
    buffers of the full width (ld = N, col0 = the shard's first column): every
    buffer ends up equal, bit for bit, to the plain entry point run on each
    shard; and the fp32 result meets the oracle's bar."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant_b200.sharding import shard_bounds, shard_groupwise

    nat, lib = _lib()
    m, n, k, g, kernel, xdt = case
    rng = np.random.default_rng(11)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    x = rng.normal(size=(m, k)).astype(np.float32)
    q = quantize_int4_groupwise(torch.from_numpy(w).cuda(), g)
    xt = torch.from_numpy(x).cuda().to(xdt)
    bias = torch.from_numpy(rng.normal(size=n).astype(np.float32)).cuda()
    ycode = {torch.float32: nat.OQ_F32, torch.bfloat16: nat.OQ_BF16}[y_dtype]
    xcode = nat.OQ_F16 if xdt == torch.float16 else nat.OQ_BF16
    sel = nat.KERNELS[kernel]
    world = 3
    bufs = [torch.full((m, n), float("nan"), device="cuda").to(y_dtype) for _ in range(world)]
    plain = torch.empty((m, n), device="cuda", dtype=y_dtype)
    stream = nat.stream_of(xt.device)
    for r in range(world):
        a, b = shard_bounds(n, world, r)
        sh = shard_groupwise(q, world, r)
        order = [bufs[(r + j) % world] for j in range(world)]
        nat.check(lib.oq_int4_linear_peers(xt.data_ptr(), xcode, sh.data.data_ptr(), sh.scales.data_ptr(),
                                           _ptrs(order), world, ycode, bias[a:b].data_ptr(), n, a, m, b - a, k, g,
                                           sel, 0, None, 0, stream))
        part = torch.empty((m, b - a), device="cuda", dtype=y_dtype)
        nat.check(lib.oq_int4_linear_ex(xt.data_ptr(), xcode, sh.data.data_ptr(), sh.scales.data_ptr(),
                                        part.data_ptr(), ycode, bias[a:b].data_ptr(), m, b - a, k, g, sel, 0, stream))
        plain[:, a:b] = part
    torch.cuda.synchronize()
    assert _take_device_error() == 0
    for buf in bufs:
        assert torch.equal(buf.view(torch.int16 if y_dtype != torch.float32 else torch.int32),
                           plain.view(torch.int16 if y_dtype != torch.float32 else torch.int32))
    if y_dtype == torch.float32:
        name = "f16" if xdt == torch.float16 else "bf16"
        data, scales = q.data.cpu().numpy(), q.scales.cpu().numpy()
        ref = orc.int4_linear(x, data, scales, n, g, x_dtype=name) + bias.cpu().numpy().astype(np.float64)
        err = bufs[0].cpu().numpy().astype(np.float64) - ref
        assert np.linalg.norm(err) / np.linalg.norm(ref) <= 1e-3
        assert np.abs(err).max() <= 2e-2


def test_peers_entry_rejects_bad_columns():
    nat, lib = _lib()
    x = torch.zeros(1, 256, device="cuda", dtype=torch.float16)
    p = torch.zeros(64 * 128, device="cuda", dtype=torch.uint8)
    s = torch.ones(64, 2, device="cuda")
    y = torch.zeros(1, 100, device="cuda")
    stream = nat.stream_of(x.device)
    # columns [50, 114) do not fit a row of 100
    st = lib.oq_int4_linear_peers(x.data_ptr(), nat.OQ_F16, p.data_ptr(), s.data_ptr(), _ptrs([y]), 1, nat.OQ_F32,
                                  None, 100, 50, 1, 64, 256, 128, 0, 0, None, 0, stream)
    assert st == nat.OQ_ERR_INVALID and "col0" in nat.last_error()
    st = lib.oq_int4_linear_peers(x.data_ptr(), nat.OQ_F16, p.data_ptr(), s.data_ptr(), _ptrs([y] * 9), 9, nat.OQ_F32,
                                  None, 100, 0, 1, 64, 256, 128, 0, 0, None, 0, stream)
    assert st == nat.OQ_ERR_INVALID


def _flag_arrays(world):
    nat, _ = _lib()
    return [torch.zeros(nat.PEER_FLAG_WORDS, dtype=torch.int32, device="cuda") for _ in range(world)]


def test_peer_barrier_counts_and_signals():
    """Rank 0 of two, with rank 1's arrivals already in its array: each call
    passes, counts itself in the last word and signals both arrays."""
    nat, lib = _lib()
    flags = _flag_arrays(2)
    stream = nat.stream_of(flags[0].device)
    for epoch in (1, 2, 3):
        flags[0][1] = epoch  # "rank 1 has arrived"
        nat.check(lib.oq_peer_barrier(_ptrs(flags), 2, 0, 0, stream))
        torch.cuda.synchronize()
        assert _take_device_error() == 0
        assert int(flags[0][nat.PEER_FLAG_WORDS - 1]) == epoch
        assert int(flags[0][0]) == epoch and int(flags[1][0]) == epoch


def test_peer_barrier_gives_up_and_reports():
    """A peer that never arrives: the wait runs out after its timeout, the
    kernel returns, the device error word says 2, and the GPU stays usable."""
    nat, lib = _lib()
    flags = _flag_arrays(3)
    stream = nat.stream_of(flags[0].device)
    flags[0][2] = 1  # rank 2 arrived, rank 1 never does
    nat.check(lib.oq_peer_barrier(_ptrs(flags), 3, 0, 20_000_000, stream))  # 20 ms
    torch.cuda.synchronize()
    assert _take_device_error() == 2
    assert _take_device_error() == 0
    t = torch.arange(10, device="cuda")
    assert int(t.sum()) == 45


def _ipc_child(handle, n, queue):
    try:
        from openquant_b200 import _native as nat
        from openquant_b200.sharding import _DeviceArray

        torch.cuda.set_device(0)
        lib = nat.load()
        p = ctypes.c_void_p()
        h = (ctypes.c_uint8 * nat.PEER_HANDLE_BYTES).from_buffer_copy(handle)
        nat.check(lib.oq_peer_import(h, ctypes.byref(p)))
        t = torch.as_tensor(_DeviceArray(p.value, (n,), "<f4"), device="cuda")
        t.copy_(torch.arange(n, dtype=torch.float32, device="cuda"))
        torch.cuda.synchronize()
        nat.check(lib.oq_peer_close(p))
        queue.put("ok")
    except Exception as exc:  # report, never hang the parent
        queue.put(repr(exc))


def test_peer_buffer_export_import_across_processes():
    """A buffer from oq_peer_alloc, exported by this process, mapped and
    written by another process, read back here; freed after the other side
    closed its mapping."""
    nat, lib = _lib()
    n = 4096
    p = ctypes.c_void_p()
    nat.check(lib.oq_peer_alloc(4 * n, ctypes.byref(p)))
    try:
        from openquant_b200.sharding import _DeviceArray

        mine = torch.as_tensor(_DeviceArray(p.value, (n,), "<f4"), device="cuda")
        assert int(mine.abs().sum()) == 0  # zeroed
        h = (ctypes.c_uint8 * nat.PEER_HANDLE_BYTES)()
        nat.check(lib.oq_peer_export(p, h))
        ctx = mp.get_context("spawn")
        queue = ctx.Queue()
        proc = ctx.Process(target=_ipc_child, args=(bytes(h), n, queue))
        proc.start()
        res = queue.get(timeout=300)
        proc.join(timeout=60)
        assert res == "ok", res
        assert torch.equal(mine, torch.arange(n, dtype=torch.float32, device="cuda"))
    finally:
        torch.cuda.synchronize()
        nat.check(lib.oq_peer_free(p))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, queue):
    from datetime import timedelta

    import torch.distributed as dist

    os.environ["NCCL_NVLS_ENABLE"] = "0"
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
        errs = []
        for mode in ("p2p", "nccl"):
            lin = ShardedInt4Linear(shard_groupwise(q, world, rank), n, mode=mode)
            for xs in (x, x[:4].half().contiguous(), x[:1].half().contiguous()):
                full = int4_linear(xs, q.data, q.scales, n, g)
                for _ in range(3):  # both output buffers, and one reused
                    y = lin(xs)
                    # the local shape may take another launch shape than the
                    # full layer's: fp32 summation order only
                    errs.append((y - full).abs().max().item())
            if mode == "p2p":
                y32 = lin(x)
                yb = lin(x, out_dtype=torch.bfloat16)  # same sums, rounded once to bf16
                errs.append(0.0 if torch.equal(yb, y32.bfloat16()) else float("inf"))
            lin.close()
        owned = quantize_layers(lambda i: torch.randn(64, 256, device=dev), 5, group_size=64)
        torch.cuda.synchronize()
        code = ctypes.c_int32(-1)
        from openquant_b200 import _native as nat

        nat.check(nat.load().oq_take_device_error(ctypes.byref(code)))
        dist.destroy_process_group()
        queue.put((rank, max(errs), code.value, sorted(owned)))
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
    for rank, err, code, owned in res:
        assert isinstance(err, float), err
        assert err <= 1e-4, (rank, err)
        assert code == 0
        assert owned == [i for i in range(5) if i % 2 == rank]
