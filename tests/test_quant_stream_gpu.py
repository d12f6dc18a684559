"""Groupwise quantizer on its streaming path (K % g == 0, g a power of two in
[8, 256]): weights walked in 16 KB tiles through a shared-memory ring.  Bit
for bit against the oracle with several tiles per CTA, a partial last tile,
exact and near ties of the quotient, and every weight dtype.
"""
import numpy as np
import pytest
import torch

import oq_oracle as orc

pytestmark = pytest.mark.gpu

DTYPES = [torch.float32, torch.float16, torch.bfloat16]


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    from openquant_b200 import build

    build.build()


def _check(wt, g):
    from openquant.groupwise import quantize_int4_groupwise

    n, k = wt.shape
    q = quantize_int4_groupwise(wt.cuda(), g)
    data, scales = orc.quantize_int4_groupwise(wt.float().numpy(), g)
    got = q.data.cpu().numpy()
    bad = np.flatnonzero(got != data)
    assert bad.size == 0, f"{bad.size} packed bytes differ, first at {bad[:4]}"
    np.testing.assert_array_equal(q.scales.cpu().numpy().view(np.uint32), scales.view(np.uint32))
    assert q.scales.shape == (n, k // g)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("g", [8, 16, 32, 64, 128, 256])
def test_stream_partial_last_tile(dtype, g):
    # 53 x 1024 weights: 6.6 tiles of 2-byte weights, 13.3 of fp32.
    rng = np.random.default_rng(g)
    w = rng.normal(0, 0.05, (53, 1024)).astype(np.float32)
    w[5, 100:100 + g] = 0.0  # an all-zero group: scale 1
    w[7, :g] *= 1e-37  # subnormal weights and scale (fp16: zeros): exact IEEE path
    _check(torch.from_numpy(w).to(dtype), g)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("g", [16, 128])
def test_stream_ties_and_near_ties(dtype, g):
    # Groups whose max is 7 * 2^e make the scale 2^e, so (j + 1/2) * 2^e
    # quotients are exact ties (round half to even).  Off-tie offsets: 2^-20
    # in fp32 (a near tie only the exact path decides), 2^-8 in fp16 (the
    # finest step the format has below 8).
    rng = np.random.default_rng(7)
    n, k = 40, 2048
    w = torch.from_numpy(rng.normal(0, 1.0, (n, k)).astype(np.float32)).to(dtype).float().numpy()
    step = {torch.float32: 2.0 ** -20, torch.float16: 2.0 ** -8, torch.bfloat16: 0.0}[dtype]
    for r in range(0, n, 2):
        e = 2.0 ** int(rng.integers(-8, 4))
        for c0 in range(0, k, g):
            if rng.random() < 0.5:
                continue
            grp = (rng.integers(-7, 7, g) + 0.5).astype(np.float32)
            grp += rng.choice([0.0, step, -step], g).astype(np.float32)
            grp[int(rng.integers(0, g))] = 7.0 * (1 if rng.random() < 0.5 else -1)
            w[r, c0:c0 + g] = grp * e
    wt = torch.from_numpy(w).to(dtype)
    assert np.array_equal(wt.double().numpy(), w.astype(np.float64)), "test values must be exact in the dtype"
    _check(wt, g)


@pytest.mark.parametrize("dtype,g", [(torch.bfloat16, 128), (torch.float16, 32), (torch.float32, 64)])
def test_stream_many_tiles_per_cta(dtype, g):
    # 4100 x 8192 weights: thousands of tiles, so every CTA wraps its ring
    # several times; outliers at 10 sigma make some groups' scales large.
    gen = torch.Generator().manual_seed(11)
    w = torch.randn(4100, 8192, generator=gen).mul_(0.02)
    idx = torch.randint(0, w.numel(), (w.numel() // 1000,), generator=gen)
    w.view(-1)[idx] = 0.2
    _check(w.to(dtype), g)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("bad", [float("nan"), float("inf"), float("-inf")])
def test_stream_nonfinite_rejected(dtype, bad):
    from openquant.groupwise import quantize_int4_groupwise

    w = torch.randn(300, 1024).mul_(0.02)
    w[299, 1023] = bad  # the last weight of the last (partial) tile
    with pytest.raises(ValueError, match="finite"):
        quantize_int4_groupwise(w.to(dtype).cuda(), 64)
    w[299, 1023] = 0.0
    w[0, 0] = bad  # the first weight
    with pytest.raises(ValueError, match="finite"):
        quantize_int4_groupwise(w.to(dtype).cuda(), 128)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_stream_16bit_fast_path_exhaustive(dtype):
    """Every (max, weight) pair of finite 16-bit values with |weight| <= max:
    one row per max m, laid out as 258 groups of 256 (m, then 255 weight bit
    patterns; patterns above m become 0), so the row covers all 65536
    patterns.  The streaming kernel (16-byte-aligned weights) must give the
    same bytes and scales as the per-lane IEEE kernel, which the dispatcher
    takes for weights that are not 16-byte aligned."""
    from openquant_b200 import _native as nat

    lib = nat.load()
    code = {torch.bfloat16: nat.OQ_BF16, torch.float16: nat.OQ_F16}[dtype]
    m_top = 0x7F7F if dtype == torch.bfloat16 else 0x7BFF  # largest finite
    g, groups = 256, 258
    k = g * groups
    dev = torch.device("cuda")
    slots = torch.arange(groups * (g - 1), device=dev, dtype=torch.int32)
    slots = torch.where(slots < 65536, slots, torch.zeros_like(slots))
    mismatched = 0
    for m0 in range(1, m_top + 1, 2048):
        m = torch.arange(m0, min(m0 + 2048, m_top + 1), device=dev, dtype=torch.int32)
        n = m.numel()
        wb = slots.unsqueeze(0).expand(n, -1)
        wb = torch.where((wb & 0x7FFF) <= m.unsqueeze(1), wb, torch.zeros_like(wb)).view(n, groups, g - 1)
        bits = torch.cat([m.view(n, 1, 1).expand(n, groups, 1), wb], dim=2).reshape(n, k)
        w = (bits - ((bits & 0x8000) << 1)).to(torch.int16).view(dtype)  # the 16-bit patterns
        shifted = torch.empty(n * k + 8, dtype=dtype, device=dev)
        shifted[1:n * k + 1] = w.view(-1)
        outs = []
        for src in (w, shifted[1:]):
            packed = torch.empty(n * k // 2, dtype=torch.uint8, device=dev)
            scales = torch.empty(n, groups, dtype=torch.float32, device=dev)
            flag = torch.zeros(1, dtype=torch.int32, device=dev)
            nat.check(lib.oq_quant_int4_group(src.data_ptr(), code, n, k, g, nat.ptr(packed), nat.ptr(scales),
                                              nat.ptr(flag), nat.stream_of(dev)))
            assert int(flag.item()) == 0
            outs.append((packed, scales))
        assert shifted[1:].data_ptr() % 16 != 0 and w.data_ptr() % 16 == 0
        assert torch.equal(outs[0][1].view(torch.int32), outs[1][1].view(torch.int32)), f"scales differ near max {m0:#x}"
        mismatched += int((outs[0][0] != outs[1][0]).sum())
        del w, shifted, outs, bits, wb
    assert mismatched == 0, f"{mismatched} packed bytes differ"


# ------------------------------------------------------------- per-row --


def _check_rowwise(wt, bits):
    from openquant.quantization import quantize

    q = quantize(wt.cuda(), bits)
    data, scales = orc.quantize(wt.float().numpy(), bits)
    got = q.data.cpu().numpy().reshape(-1)
    bad = np.flatnonzero(got != data.reshape(-1))
    assert bad.size == 0, f"{bad.size} bytes differ, first at {bad[:4]}"
    np.testing.assert_array_equal(q.scales.cpu().numpy().reshape(-1).view(np.uint32),
                                  scales.reshape(-1).view(np.uint32))


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("shape", [(3001, 8), (700, 64), (515, 1000), (300, 8192), (40, 28672), (9, 51200)])
def test_rowwise_stream_shapes_vs_oracle(dtype, bits, shape):
    # Stages of many short rows (K = 8 .. 1000: up to 1024 rows per 16 KB
    # stage, partial last stage), one row per stage (K = 8192: 16 KB of 2-byte
    # weights) and long rows (K = 28672, 51200: 56 and 100 KB of 2-byte
    # weights; fp32 rows above 100 KB take the two-pass kernel).
    rng = np.random.default_rng(shape[0] + shape[1] + bits)
    w = rng.normal(0, 0.05, shape).astype(np.float32)
    w[1, :] = 0.0  # zero row: scale 1
    w[2, :] *= 1e-37  # subnormal row (fp16: zero)
    _check_rowwise(torch.from_numpy(w).to(dtype), bits)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("bits", [8, 4])
def test_rowwise_stream_ties(dtype, bits):
    # Rows whose max is qmax * 2^e have scale 2^e, so (j + 1/2) * 2^e are
    # exact ties; fp32 / fp16 rows also get near ties (see the groupwise test).
    qmax = 127 if bits == 8 else 7
    rng = np.random.default_rng(bits)
    n, k = 64, 4096
    w = torch.from_numpy(rng.normal(0, 1.0, (n, k)).astype(np.float32)).to(dtype).float().numpy()
    # Off-tie steps exact up to |j + 1/2| = qmax - 1/2 in each format.
    step = {torch.float32: 2.0 ** (-20 if bits == 4 else -16), torch.float16: 2.0 ** (-8 if bits == 4 else -3),
            torch.bfloat16: 0.0}[dtype]
    for r in range(0, n, 2):
        e = 2.0 ** int(rng.integers(-8, 2))
        row = (rng.integers(-qmax, qmax, k) + 0.5).astype(np.float32)
        row += rng.choice([0.0, step, -step], k).astype(np.float32)
        row[int(rng.integers(0, k))] = qmax
        w[r] = row * e
    wt = torch.from_numpy(w).to(dtype)
    assert np.array_equal(wt.double().numpy(), w.astype(np.float64)), "test values must be exact in the dtype"
    _check_rowwise(wt, bits)


@pytest.mark.parametrize("dtype,bits", [(torch.bfloat16, 8), (torch.float16, 8), (torch.bfloat16, 4)])
def test_rowwise_16bit_fast_path_exhaustive(dtype, bits):
    """Every (max, weight) pair of finite 16-bit values with |weight| <= max,
    per-row: two rows of 32768 per max m (m, then the bit patterns; patterns
    above m become 0).  The streaming kernel (16-byte-aligned weights) must
    give the same bytes and scales as the two-pass IEEE kernel, which the
    dispatcher takes for weights that are not 16-byte aligned."""
    from openquant_b200 import _native as nat

    lib = nat.load()
    code = {torch.bfloat16: nat.OQ_BF16, torch.float16: nat.OQ_F16}[dtype]
    fn = lib.oq_quant_int8_rowwise if bits == 8 else lib.oq_quant_int4_rowwise
    m_top = 0x7F7F if dtype == torch.bfloat16 else 0x7BFF
    k = 32768
    dev = torch.device("cuda")
    pat = torch.arange(65536, device=dev, dtype=torch.int32).view(2, k)[:, :k - 1]  # 0x7FFF, 0xFFFF (NaN) left out
    mismatched = 0
    for m0 in range(1, m_top + 1, 1024):
        m = torch.arange(m0, min(m0 + 1024, m_top + 1), device=dev, dtype=torch.int32)
        nm = m.numel()
        wb = pat.unsqueeze(0).expand(nm, -1, -1)
        wb = torch.where((wb & 0x7FFF) <= m.view(nm, 1, 1), wb, torch.zeros_like(wb))
        bits_ = torch.cat([m.view(nm, 1, 1).expand(nm, 2, 1), wb], dim=2).reshape(2 * nm, k)
        w = (bits_ - ((bits_ & 0x8000) << 1)).to(torch.int16).view(dtype)
        n = 2 * nm
        shifted = torch.empty(n * k + 8, dtype=dtype, device=dev)
        shifted[1:n * k + 1] = w.view(-1)
        outs = []
        for src in (w, shifted[1:]):
            q = torch.empty(n * k // (1 if bits == 8 else 2), dtype=torch.uint8, device=dev)
            scales = torch.empty(n, dtype=torch.float32, device=dev)
            nat.check(fn(src.data_ptr(), code, n, k, nat.ptr(q), nat.ptr(scales), nat.stream_of(dev)))
            outs.append((q, scales))
        assert torch.equal(outs[0][1].view(torch.int32), outs[1][1].view(torch.int32)), f"scales differ near max {m0:#x}"
        mismatched += int((outs[0][0] != outs[1][0]).sum())
        del w, shifted, outs, bits_, wb
    assert mismatched == 0, f"{mismatched} bytes differ"
