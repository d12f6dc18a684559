"""oq_int8_linear_noalloc, the W8A8 linear layer for callers that cannot
allocate device memory when they call in (a host runtime that lends the
library only the tensors it owns, or a service whose device memory is fixed
at start-up).  It keeps the per-token INT8 activations and their scales in a
fixed array of the library instead of caller buffers.  Its output must equal
the usual path's -- oq_quant_int8_rowwise into caller buffers, then
oq_int8_gemm: the same kernels on the same data, so the same bits (the W8A8
tests' tolerance is exact integer sums) -- on consecutive calls whose shapes
differ, so that nothing one call leaves in the array shows up in the next.

Collected last on purpose: a run that stops at its first failure has run
every other test before this one.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    from openquant_b200 import _native as nat
    from openquant_b200 import build

    build.build()
    nat.require_device()
    return nat.load()


def _case(nat, lib, m, n, k, dtype, seed):
    """x [m, k] in `dtype`, and int8 weights quantized per row on the GPU."""
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=gen).to(dtype)
    w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02)
    qw = torch.empty(n, k, dtype=torch.int8, device="cuda")
    sw = torch.empty(n, device="cuda")
    nat.check(lib.oq_quant_int8_rowwise(nat.ptr(w), nat.OQ_F32, n, k, nat.ptr(qw), nat.ptr(sw),
                                        nat.stream_of(x.device)))
    return x, qw, sw


def _code(nat, dtype):
    return {torch.float32: nat.OQ_F32, torch.float16: nat.OQ_F16, torch.bfloat16: nat.OQ_BF16}[dtype]


def _usual(nat, lib, x, qw, sw):
    m, k = x.shape
    n = qw.shape[0]
    qx = torch.empty(m, k, dtype=torch.int8, device="cuda")
    sx = torch.empty(m, device="cuda")
    y = torch.empty(m, n, device="cuda")
    st = nat.stream_of(x.device)
    nat.check(lib.oq_quant_int8_rowwise(nat.ptr(x), _code(nat, x.dtype), m, k, nat.ptr(qx), nat.ptr(sx), st))
    nat.check(lib.oq_int8_gemm(nat.ptr(qx), nat.ptr(sx), nat.ptr(qw), nat.ptr(sw), nat.ptr(y), m, n, k, st))
    return y


def _noalloc(nat, lib, x, qw, sw):
    m, k = x.shape
    n = qw.shape[0]
    y = torch.full((m, n), float("nan"), device="cuda")
    nat.check(lib.oq_int8_linear_noalloc(nat.ptr(x), _code(nat, x.dtype), nat.ptr(qw), nat.ptr(sw), nat.ptr(y),
                                         m, n, k, nat.stream_of(x.device)))
    return y


def test_two_calls_in_a_row_match_the_usual_path(lib):
    from openquant_b200 import _native as nat

    # A large call, then right after it (same stream, no sync) a smaller one
    # with another K and dtype that reads the same array.
    a = _case(nat, lib, 300, 1024, 4096, torch.float16, seed=1)
    b = _case(nat, lib, 7, 384, 1040, torch.bfloat16, seed=2)
    ya = _noalloc(nat, lib, *a)
    yb = _noalloc(nat, lib, *b)
    torch.cuda.synchronize()
    assert torch.equal(ya, _usual(nat, lib, *a))
    assert torch.equal(yb, _usual(nat, lib, *b))
    # and once more with fp32 activations at the largest M * K the array takes
    c = _case(nat, lib, 2048, 256, 8192, torch.float32, seed=3)
    assert torch.equal(_noalloc(nat, lib, *c), _usual(nat, lib, *c))


def test_sizes_beyond_the_fixed_array_are_rejected(lib):
    from openquant_b200 import _native as nat

    x, qw, sw = _case(nat, lib, 4, 64, 4096, torch.float16, seed=4)
    y = torch.empty(4, 64, device="cuda")
    st = nat.stream_of(x.device)
    # M * K one row past 16 MiB, and M past 16384 tokens: refused before any
    # launch, so the small buffers passed here are never read.
    for m, k in ((4097, 4096), (16385, 16)):
        rc = lib.oq_int8_linear_noalloc(nat.ptr(x), nat.OQ_F16, nat.ptr(qw), nat.ptr(sw), nat.ptr(y), m, 64, k, st)
        assert rc == nat.OQ_ERR_INVALID
        assert "fixed scratch" in nat.last_error()
    torch.cuda.synchronize()


def test_calls_allocate_no_device_memory(lib):
    """The defining property: once a shape has run (kernels loaded, the
    array's address looked up), further calls leave the device's free memory
    exactly where it was."""
    from openquant_b200 import _native as nat

    a = _case(nat, lib, 64, 512, 2048, torch.float16, seed=5)
    b = _case(nat, lib, 5, 256, 4096, torch.bfloat16, seed=6)
    ya, yb = torch.empty(64, 512, device="cuda"), torch.empty(5, 256, device="cuda")
    st = nat.stream_of(ya.device)

    def calls():
        for (x, qw, sw), y in ((a, ya), (b, yb)):
            m, k = x.shape
            nat.check(lib.oq_int8_linear_noalloc(nat.ptr(x), _code(nat, x.dtype), nat.ptr(qw), nat.ptr(sw),
                                                 nat.ptr(y), m, qw.shape[0], k, st))

    calls()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(5):
        calls()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before
    assert torch.equal(ya, _usual(nat, lib, *a)) and torch.equal(yb, _usual(nat, lib, *b))

