"""int4_linear vs the oracle's dequantise-then-matmul.

The oracle rounds the dequantized weights to x's dtype before the product,
as the reference kernel and its test do (triton_int4.py:62-65,
tests/test_triton_int4.py:45-51), and sums in fp64.  Tolerances: rel-L2
<= 1e-3 and max-abs <= 2e-2 (the bar for this path), and the reference
test's own assert_close(rtol=0.02, atol=0.02).
"""
import numpy as np
import pytest
import torch

import oq_oracle as orc

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3
MAX_ABS = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    from openquant_b200 import build

    build.build()


def make_case(m, n, k, g, dtype, seed=42, w_sigma=1.0):
    from openquant.groupwise import quantize_int4_groupwise

    rng = np.random.default_rng(seed)
    w = rng.normal(0, w_sigma, (n, k)).astype(np.float32)
    x = rng.normal(size=(m, k)).astype(np.float32)
    q = quantize_int4_groupwise(w, g)
    xt = torch.from_numpy(x).cuda().to(dtype)
    return x, q, xt


def assert_no_device_error():
    import ctypes

    from openquant_b200 import _native as nat

    code = ctypes.c_int32(-1)
    nat.check(nat.load().oq_take_device_error(ctypes.byref(code)))
    assert code.value == 0, f"kernel reported device error {code.value}"


def check_against_oracle(y, x, q, g, dtype):
    assert_no_device_error()
    name = "f16" if dtype == torch.float16 else "bf16"
    ref = orc.int4_linear(x, q.data, q.scales, q.shape[0], g, x_dtype=name)
    got = y.cpu().numpy()
    assert got.shape == ref.shape and np.isfinite(got).all()
    err = got.astype(np.float64) - ref
    rel = np.linalg.norm(err) / max(np.linalg.norm(ref), 1e-30)
    assert rel <= REL_L2, rel
    assert np.abs(err).max() <= MAX_ABS, np.abs(err).max()
    torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(ref), rtol=0.02, atol=0.02)
    return rel


@pytest.mark.parametrize("shape", [(3, 7, 65, 16), (16, 32, 128, 32), (33, 55, 79, 16)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_reference_test_shapes(shape, dtype):
    from openquant.triton_int4 import int4_linear

    m, n, k, g = shape
    x, q, xt = make_case(m, n, k, g, dtype)
    y = int4_linear(xt, torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda(), n, g)
    assert y.dtype == torch.float32 and y.shape == (m, n)
    check_against_oracle(y, x, q, g, dtype)


@pytest.mark.parametrize("cfg", [8, 9, 10, 12, 13, 8 | 16, 9 | 16, 12 | 16, 13 | 16, 10 | 32, 12 | 32, 13 | 32])
@pytest.mark.parametrize("shape", [(1, 4096, 4096, 128), (1, 1000, 11008, 128), (16, 300, 4096, 64),
                                   (9, 77, 1000, 32), (2, 4097, 1152, 256), (1, 16, 8, 32), (5, 40, 3000, 128)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tma_gemv_vs_oracle(shape, dtype, cfg):
    """The TMA-fed GEMVs (configs 8-10 persistent, 12 one CTA per tile, 13
    one CTA per SM owning two tiles;
    | 16 = exact rounding, | 32 = static weights streamed before the wait on
    the previous kernel)."""
    from openquant_b200 import _native as nat

    m, n, k, g = shape
    if g > 32 * (16 if (cfg & 15) == 9 else 8):
        pytest.skip("group too large for this config")
    x, q, xt = make_case(m, n, k, g, dtype, seed=m + n + k, w_sigma=0.02)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    y = torch.empty(m, n, device="cuda")
    code = nat.OQ_F16 if dtype == torch.float16 else nat.OQ_BF16
    st = nat.load().oq_int4_linear(nat.ptr(xt), code, nat.ptr(p), nat.ptr(s), nat.ptr(y), m, n, k, g, 1, cfg,
                                   nat.stream_of(xt.device))
    if st != 0 and (cfg & 15) >= 10 and "does not take this shape" in nat.last_error():
        pytest.skip("shape outside this config's shared-memory plan")
    nat.check(st)
    check_against_oracle(y, x, q, g, dtype)


@pytest.mark.parametrize("shape", [(1, 4096, 4096, 128), (4, 4096, 12288, 128), (16, 300, 4096, 64),
                                   (1, 1000, 11008, 128)])
def test_static_weights_same_result_and_ordering(shape):
    """OQ_CONFIG_STATIC_WEIGHTS changes only when the weights are streamed:
    the output is bit-identical to the default launch, for every GEMV config
    that takes the shape; and a GEMV right after the quantizer that writes its
    weights (default launch: no early read) sees the new weights."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear
    from openquant_b200 import _native as nat

    m, n, k, g = shape
    x, q, xt = make_case(m, n, k, g, torch.float16, seed=n + k, w_sigma=0.02)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    lib = nat.load()
    for cfg in (0, 1, 8, 10, 12, 13):
        outs = []
        for flag in (0, nat.CONFIG_STATIC_WEIGHTS):
            y = torch.full((m, n), float("nan"), device="cuda")
            st = lib.oq_int4_linear(nat.ptr(xt), nat.OQ_F16, nat.ptr(p), nat.ptr(s), nat.ptr(y), m, n, k, g, 1,
                                    cfg | flag, nat.stream_of(xt.device))
            if st != 0:
                assert "does not take this shape" in nat.last_error()
                break
            outs.append(y)
        if len(outs) == 2:
            assert torch.equal(outs[0], outs[1]), cfg
    # quantize -> GEMV on one stream, back to back, three times with new weights
    gen = torch.Generator(device="cuda").manual_seed(3)
    for _ in range(3):
        w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02).half()
        qg = quantize_int4_groupwise(w, g)
        y = int4_linear(xt, qg.data, qg.scales, n, g)
        torch.cuda.synchronize()
        y_ref = int4_linear(xt, qg.data.clone(), qg.scales.clone(), n, g)
        assert torch.equal(y, y_ref)


GEMV_SHAPES = [
    (1, 16, 32, 32), (1, 17, 64, 32), (2, 48, 96, 32), (4, 100, 200, 64), (8, 33, 256, 128), (9, 64, 1024, 128),
    (16, 4096, 4096, 128), (1, 4096, 4096, 128), (5, 31, 160, 32), (16, 8, 8, 32), (1, 1, 8, 32), (64, 70, 384, 128),
    (40, 130, 520, 64), (1, 1000, 11008, 128), (16, 256, 11008, 128), (48, 64, 2048, 64), (3, 40, 200, 32),
]


@pytest.mark.parametrize("kernel", ["gemv", "simt", None])
@pytest.mark.parametrize("shape", GEMV_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_decode_kernels_vs_oracle(shape, dtype, kernel):
    from openquant.triton_int4 import int4_linear

    m, n, k, g = shape
    if kernel == "simt" and m * n * k > 2e8:
        pytest.skip("SIMT kernel checked on smaller shapes")
    x, q, xt = make_case(m, n, k, g, dtype, seed=m * 7 + n + k, w_sigma=0.02)
    y = int4_linear(xt, torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda(), n, g, kernel=kernel)
    check_against_oracle(y, x, q, g, dtype)


@pytest.mark.parametrize("shape", [(3, 20, 30, 2), (4, 9, 33, 6), (17, 40, 100, 10), (2, 16, 200, 16), (1, 5, 7, 8)])
def test_simt_any_group_vs_oracle(shape):
    from openquant.triton_int4 import int4_linear

    m, n, k, g = shape
    for dtype in (torch.float16, torch.bfloat16):
        x, q, xt = make_case(m, n, k, g, dtype)
        y = int4_linear(xt, torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda(), n, g)
        check_against_oracle(y, x, q, g, dtype)


def test_llama2_7b_decode_layer_set():
    """M in {1, 4, 16} over the Llama-2-7B layer set, g = 128, fp16."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear

    for li, (k, n) in enumerate([(4096, 12288), (4096, 4096), (4096, 22016), (11008, 4096)]):
        gen = torch.Generator(device="cuda").manual_seed(100 + li)
        w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02).half()
        q = quantize_int4_groupwise(w, 128)
        wd = orc.dequantize_int4_groupwise(q.data.cpu().numpy(), q.scales.cpu().numpy(), (n, k), 128)
        w16 = torch.from_numpy(orc.round_to_dtype(wd, "f16")).cuda().double()
        for m in (1, 4, 16):
            x = torch.randn(m, k, device="cuda", generator=gen).half()
            y = int4_linear(x, q.data, q.scales, n, 128)
            ref = x.double() @ w16.T
            err = y.double() - ref
            assert (err.norm() / ref.norm()).item() <= REL_L2
            assert err.abs().max().item() <= MAX_ABS


def test_out_argument_and_errors():
    from openquant.triton_int4 import int4_linear

    x, q, xt = make_case(4, 64, 128, 32, torch.float16)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    out = torch.full((4, 64), float("nan"), device="cuda")
    y = int4_linear(xt, p, s, 64, 32, out=out)
    assert y.data_ptr() == out.data_ptr()
    check_against_oracle(y, x, q, 32, torch.float16)
    with pytest.raises(ValueError, match="scales shape"):
        int4_linear(xt, p, s[:, :1].contiguous(), 64, 32)
    with pytest.raises(ValueError, match="packed weight count"):
        int4_linear(xt, p[:-1], s, 64, 32)
    with pytest.raises(ValueError, match="contiguous"):
        int4_linear(xt.t().contiguous().t(), p, s, 64, 32)
    with pytest.raises(ValueError, match="Group size"):
        int4_linear(xt, p, s, 64, 3)
    with pytest.raises(ValueError, match="uint8"):
        int4_linear(xt, p.to(torch.int8), s, 64, 32)
    with pytest.raises(ValueError, match="float32"):
        int4_linear(xt, p, s.double(), 64, 32)
    with pytest.raises(ValueError):
        int4_linear(xt, p, s, 64, 32, kernel="gemv", out=torch.empty(3, 3, device="cuda"))


def test_deterministic_repeat():
    from openquant.triton_int4 import int4_linear

    x, q, xt = make_case(16, 512, 4096, 128, torch.bfloat16)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    a = int4_linear(xt, p, s, 512, 128)
    b = int4_linear(xt, p, s, 512, 128)
    assert torch.equal(a, b)


PREFILL_SHAPES = [
    (64, 128, 64, 32), (100, 200, 136, 64), (256, 256, 1024, 128), (300, 129, 520, 32), (17, 1000, 4096, 128),
    (512, 1024, 2048, 128), (513, 384, 8192, 128), (1024, 128, 200, 64),
    # large N at M >= 1024: the wide-tile kernel (two accumulators of NB rows),
    # ragged in M and N
    (1500, 20000, 256, 32), (2050, 18000, 512, 128), (4097, 9000, 256, 64),
]


@pytest.mark.parametrize("shape", PREFILL_SHAPES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prefill_tcgen05_vs_oracle(shape, dtype):
    """The tcgen05/TMEM GEMM against the oracle (ragged M, N, K; g 32..128;
    256-row tiles, and the wide tiles the launcher picks for large M and N)."""
    from openquant.triton_int4 import int4_linear

    m, n, k, g = shape
    x, q, xt = make_case(m, n, k, g, dtype, seed=m + 3 * n + k, w_sigma=0.02)
    y = int4_linear(xt, torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda(), n, g, kernel="tcgen05")
    check_against_oracle(y, x, q, g, dtype)


def test_prefill_tcgen05_llama70b_shape_sampled():
    """M = 2048, (K, N) = (8192, 28672) at bf16: compare sampled outputs with
    an fp64 product of the exactly-rounded weights."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear

    m, k, n, g = 2048, 8192, 28672, 128
    gen = torch.Generator(device="cuda").manual_seed(7)
    w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02).to(torch.bfloat16)
    q = quantize_int4_groupwise(w, g)
    del w
    x = torch.randn(m, k, device="cuda", generator=gen).to(torch.bfloat16)
    y = int4_linear(x, q.data, q.scales, n, g)
    assert_no_device_error()
    rows = torch.arange(0, n, 97, device="cuda")
    packed = q.data.view(n, k // 2)[rows].cpu().numpy().reshape(-1)
    sc = q.scales[rows].cpu().numpy()
    wr = orc.round_to_dtype(orc.dequantize_int4_groupwise(packed, sc, (len(rows), k), g), "bf16")
    ref = x.double() @ torch.from_numpy(wr).cuda().double().T
    got = y[:, rows].double()
    err = got - ref
    assert (err.norm() / ref.norm()).item() <= REL_L2
    assert err.abs().max().item() <= MAX_ABS


@pytest.mark.parametrize("kernel", ["gemv", "simt", "tcgen05", None])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(48, 512, 128), (33, 256, 64), (40, 96, 32)])
def test_weight_rounding_is_bit_exact(shape, dtype, kernel):
    """One-hot activation rows: y[m, n] = x[m, k_m] * W[n, k_m] with x = 1, a
    single exact product, so y must equal round_x(fl32(q * s)) bit for bit
    (the weight rounding of triton_int4.py:62-65) for every column probed."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear
    from conftest import assert_float_bits_equal

    n, k, g = shape
    m = {"simt": 16, "tcgen05": 256}.get(kernel, 64)
    rng = np.random.default_rng(n + k + g)
    w = rng.normal(0, 0.05, (n, k)).astype(np.float32)
    w[:, ::7] *= 1e-3  # small groups exercise other exponents
    q = quantize_int4_groupwise(w, g)
    name = "f16" if dtype == torch.float16 else "bf16"
    wref = orc.round_to_dtype(orc.dequantize_int4_groupwise(q.data, q.scales, (n, k), g), name)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    for start in range(0, k, m):
        cols = np.arange(start, min(k, start + m))
        x = np.zeros((len(cols), k), np.float32)
        x[np.arange(len(cols)), cols] = 1.0
        y = int4_linear(torch.from_numpy(x).cuda().to(dtype), p, s, n, g, kernel=kernel, exact_rounding=True)
        assert_float_bits_equal(y.cpu().numpy(), wref[:, cols].T.copy(), f"cols {start}")


@pytest.mark.parametrize("shape", [(1, 4096, 4096), (4, 4096, 22016), (16, 11008, 4096), (3, 1024, 512), (64, 256, 1024)])
def test_fp16_scale_after_vs_exact_rounding(shape):
    """fp16 GEMV default for M <= 16 (exact integer nibbles, fp32 group scale
    applied to the group's partial sum) vs the reference's per-weight fp16
    rounding: both within the parity tolerance of the oracle, and the default
    is the closer of the two to the unrounded product x.(q*s)."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear

    m, k, n = shape
    gen = torch.Generator(device="cuda").manual_seed(m + k + n)
    w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02)
    q = quantize_int4_groupwise(w, 128)
    x = torch.randn(m, k, device="cuda", generator=gen).half()
    wd = orc.dequantize_int4_groupwise(q.data.cpu().numpy(), q.scales.cpu().numpy(), (n, k), 128)
    ref = x.double() @ torch.from_numpy(orc.round_to_dtype(wd, "f16")).cuda().double().T
    true = x.double() @ torch.from_numpy(wd).cuda().double().T
    fast = int4_linear(x, q.data, q.scales, n, 128).double()
    exact = int4_linear(x, q.data, q.scales, n, 128, exact_rounding=True).double()
    for y in (fast, exact):
        assert ((y - ref).norm() / ref.norm()).item() <= REL_L2
        assert (y - ref).abs().max().item() <= MAX_ABS
    assert ((exact - ref).norm() / ref.norm()).item() < 1e-5
    if m <= 16:  # scale-after path: closer to the unrounded product
        assert (fast - true).norm().item() < (exact - true).norm().item()
    else:  # M > 16 (the tcgen05 GEMM) uses the exact rounding
        assert ((fast - exact).norm() / exact.norm()).item() < 1e-5


@pytest.mark.parametrize("kernel", ["gemv", "simt", "tcgen05", None])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 4096, 4096, 128), (5, 300, 1024, 64), (300, 640, 1024, 128),
                                   (1100, 9000, 256, 128)])  # the last: wide GEMM tiles
def test_fused_bias_and_output_dtype(shape, out_dtype, kernel):
    """The fused epilogue adds the bias in fp32 and rounds once, exactly as
    (fp32 result + bias).to(dtype) does."""
    from openquant.triton_int4 import int4_linear

    m, n, k, g = shape
    if kernel == "gemv" and m > 64:
        pytest.skip("GEMV takes M <= 64")
    x, q, xt = make_case(m, n, k, g, torch.float16, seed=m + n, w_sigma=0.02)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    bias = torch.randn(n, device="cuda")
    y32 = int4_linear(xt, p, s, n, g, kernel=kernel)
    y = int4_linear(xt, p, s, n, g, kernel=kernel, bias=bias, out_dtype=out_dtype)
    assert y.dtype == out_dtype and y.shape == (m, n)
    assert torch.equal(y, (y32 + bias).to(out_dtype))
    out = torch.empty(m, n, dtype=out_dtype, device="cuda")
    assert int4_linear(xt, p, s, n, g, kernel=kernel, bias=bias, out=out) is out
    assert torch.equal(out, y)
    # and directly against the oracle: (x . W^T + bias) within the parity bar,
    # plus the output type's own rounding (half an ulp: 2^-11 fp16, 2^-8 bf16)
    ref = orc.int4_linear(x, q.data, q.scales, n, g, x_dtype="f16") + bias.cpu().double().numpy()
    rnd = {torch.float32: 0.0, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}[out_dtype]
    err = y.double().cpu().numpy() - ref
    assert np.linalg.norm(err) / np.linalg.norm(ref) <= REL_L2 + rnd
    assert (np.abs(err) <= MAX_ABS + rnd * np.abs(ref)).all()


def test_fused_epilogue_every_gemv_config():
    from openquant_b200 import _native as nat

    m, n, k, g = 1, 4096, 4096, 128
    x, q, xt = make_case(m, n, k, g, torch.float16, seed=9, w_sigma=0.02)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    bias = torch.randn(n, device="cuda")
    lib = nat.load()
    for cfg in (0, 1, 8, 9, 10, 12, 13, 13 | 32):
        y32 = torch.empty(m, n, device="cuda")
        nat.check(lib.oq_int4_linear(nat.ptr(xt), nat.OQ_F16, nat.ptr(p), nat.ptr(s), nat.ptr(y32), m, n, k, g, 1,
                                     cfg, nat.stream_of(xt.device)))
        yb = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        nat.check(lib.oq_int4_linear_ex(nat.ptr(xt), nat.OQ_F16, nat.ptr(p), nat.ptr(s), nat.ptr(yb), nat.OQ_BF16,
                                        nat.ptr(bias), m, n, k, g, 1, cfg, nat.stream_of(xt.device)))
        assert torch.equal(yb, (y32 + bias).to(torch.bfloat16)), cfg


@pytest.mark.parametrize("shape", [(1, 4096, 4096, 128), (3, 11008, 4096, 128), (16, 1000, 2048, 64), (1, 24, 512, 32)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_silu_gate_fusion_matches_two_products(shape, dtype):
    """silu_gate over the [gate; up] stack equals silu(gate) * up from two
    launches of the same GEMV config (identical sums; silu from the GPU's
    expf vs torch's sigmoid in fp64: within a few ulp); the Python API's
    automatic choice is that same config."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear
    from openquant_b200 import _native as nat

    m, n, k, g = shape
    gen = torch.Generator(device="cuda").manual_seed(n + k)
    w = torch.randn(2 * n, k, device="cuda", generator=gen).mul_(0.02).to(dtype)
    q = quantize_int4_groupwise(w, g)
    x = torch.randn(m, k, device="cuda", generator=gen).to(dtype)
    code = nat.OQ_F16 if dtype == torch.float16 else nat.OQ_BF16
    lib = nat.load()
    half = q.data.numel() // 2

    def run(packed, scales, out_cols, cfg):
        y = torch.empty(m, out_cols, device="cuda")
        nat.check(lib.oq_int4_linear(nat.ptr(x), code, nat.ptr(packed), nat.ptr(scales), nat.ptr(y), m, out_cols, k,
                                     g, 1, cfg, nat.stream_of(x.device)))
        return y

    # the automatic choice: the first of 10 (M <= 8, K <= 4096), 9, 8 that
    # takes the shape (the default rounding up to M = 16)
    for cfg in ([10, 9, 8] if m <= 8 and k <= 4096 else [9, 8]):
        try:
            gate = run(q.data[:half], q.scales[:n], n, cfg)
            break
        except ValueError:
            continue
    else:
        pytest.fail("no TMA GEMV config takes this shape")
    up = run(q.data[half:], q.scales[n:], n, cfg)
    fused = run(q.data, q.scales, n, cfg | nat.CONFIG_SILU_GATE)
    ref = (gate.double() * torch.sigmoid(gate.double())) * up.double()
    err = (fused.double() - ref).abs()
    assert float((err - 2e-6 * ref.abs()).max()) <= 1e-6, float(err.max())
    y = int4_linear(x, q.data, q.scales, n, g, silu_gate=True)
    assert y.shape == (m, n) and torch.equal(y, fused)
    # directly against the oracle: silu(gate) * up from the oracle's two
    # products in fp64.  Each product meets the parity bar (max-abs eps =
    # 2e-2), so to first order |fused - ref| <= eps * (|silu'(g)| |u| +
    # |silu(g)|), with |silu'| <= 1.1.
    name = "f16" if dtype == torch.float16 else "bf16"
    data, scales = q.data.cpu().numpy(), q.scales.cpu().numpy()
    xf = x.float().cpu().numpy()
    g_ref = orc.int4_linear(xf, data[:half], scales[:n], n, g, x_dtype=name)
    u_ref = orc.int4_linear(xf, data[half:], scales[n:], n, g, x_dtype=name)
    silu = g_ref / (1.0 + np.exp(-g_ref))
    ref_o = silu * u_ref
    err_o = fused.double().cpu().numpy() - ref_o
    assert (np.abs(err_o) <= MAX_ABS * (1.1 * np.abs(u_ref) + np.abs(silu)) + 1e-6).all()
    assert np.linalg.norm(err_o) / np.linalg.norm(ref_o) <= 2 * REL_L2
    yb = int4_linear(x, q.data, q.scales, n, g, silu_gate=True, out_dtype=torch.bfloat16)
    assert torch.equal(yb, fused.to(torch.bfloat16))
    with pytest.raises(ValueError):
        int4_linear(x, q.data, q.scales, n, g, silu_gate=True, bias=torch.zeros(n, device="cuda"))


def test_tile_table_entry_outside_its_plan_falls_back(monkeypatch):
    """A tuned table entry holds for a whole batch-size bucket; when its
    launch shape rejects the call (here the tile GEMV, which needs KP <=
    4096, given K = 8192) int4_linear runs the library's automatic choice
    instead of failing, with the same result."""
    from openquant.triton_int4 import int4_linear
    from openquant_b200 import _native as nat
    from openquant_b200 import tile_table

    m, n, k, g = 4, 256, 8192, 128
    x, q, xt = make_case(m, n, k, g, torch.float16, seed=11, w_sigma=0.02)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    ref = int4_linear(xt, p, s, n, g)
    monkeypatch.setattr(tile_table, "lookup", lambda *a: (nat.KERNELS["gemv"], 12))
    y = int4_linear(xt, p, s, n, g)
    assert torch.equal(y, ref)
    check_against_oracle(y, x, q, g, torch.float16)



@pytest.mark.parametrize("case", [(1, 4096, 4096, 128, torch.float16, {}),
                                  (4, 4096, 12288, 128, torch.float16, {"static_weights": True}),
                                  (16, 11008, 4096, 128, torch.float16, {"exact_rounding": True}),
                                  (7, 1000, 300, 64, torch.bfloat16, {"out_dtype": torch.bfloat16, "bias": True}),
                                  (300, 1024, 2048, 128, torch.bfloat16, {}),
                                  (9, 200, 300, 6, torch.float16, {"kernel": "simt"})],
                         ids=lambda c: f"m{c[0]}_n{c[1]}_k{c[2]}_g{c[3]}" if isinstance(c, tuple) else "")
def test_int4_linear_layer_object_is_bit_equal(case):
    """Int4Linear (validated once) launches what int4_linear launches: the
    same output bits, call after call, with and without out=; and it refuses
    an x that does not fit its weights."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import Int4Linear, int4_linear

    m, n, k, g, dtype, opts = case
    gen = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    q = quantize_int4_groupwise(torch.randn(n, k, device="cuda", generator=gen).mul_(0.02), g)
    x = torch.randn(m, k, device="cuda", generator=gen).to(dtype)
    opts = dict(opts)
    if opts.pop("bias", False):
        opts["bias"] = torch.randn(n, device="cuda", generator=gen)
    layer = Int4Linear(q.data, q.scales, n, g, **opts)
    ref = int4_linear(x, q.data, q.scales, n, g, **opts)
    for _ in range(2):
        assert torch.equal(layer(x), ref)
    out = torch.empty_like(ref)
    assert layer(x, out=out) is out and torch.equal(out, ref)
    with pytest.raises(ValueError):
        layer(torch.zeros(m, k + g, device="cuda", dtype=dtype))
    with pytest.raises(ValueError):
        layer(x.float())
    with pytest.raises(ValueError):
        layer(x, out=torch.empty(m, n + 1, device="cuda", dtype=ref.dtype))


@pytest.mark.parametrize("case", [(1, 4096, 4096, 128, torch.float16, {"static_weights": True}),
                                  (4, 4096, 12288, 128, torch.float16, {}),
                                  (16, 11008, 4096, 128, torch.float16, {"exact_rounding": True}),
                                  (7, 1000, 300, 64, torch.bfloat16, {"out_dtype": torch.bfloat16, "bias": True}),
                                  (9, 200, 300, 6, torch.float16, {"kernel": "simt"}),
                                  (40, 512, 1024, 128, torch.bfloat16, {})],
                         ids=lambda c: f"m{c[0]}_n{c[1]}_k{c[2]}_g{c[3]}" if isinstance(c, tuple) else "")
def test_int4_linear_forward_host(case):
    """Int4Linear.forward_host (oq_int4_linear_host): x and y in page-locked
    host memory; a copy kernel brings x over the bus and the layer kernel
    writes y into host memory.  For decode shapes the output equals the
    device-buffer call's bit for bit; above M = 16 the prefill GEMM runs
    without its stream-K split and meets the oracle bar.  Pageable host memory
    and device tensors are refused."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import Int4Linear

    m, n, k, g, dtype, opts = case
    gen = torch.Generator(device="cuda").manual_seed(m * 5 + n)
    w = torch.randn(n, k, device="cuda", generator=gen).mul_(0.02)
    q = quantize_int4_groupwise(w, g)
    x = torch.randn(m, k, device="cuda", generator=gen).to(dtype)
    opts = dict(opts)
    if opts.pop("bias", False):
        opts["bias"] = torch.randn(n, device="cuda", generator=gen)
    layer = Int4Linear(q.data, q.scales, n, g, **opts)
    ref = layer(x).cpu()
    x_host = x.cpu().pin_memory()
    for _ in range(2):
        got = layer.forward_host(x_host)
        assert got.is_pinned() and got.dtype == ref.dtype and got.shape == ref.shape
        if m <= 16:
            assert torch.equal(got, ref)
    out = torch.empty(ref.shape, dtype=ref.dtype, pin_memory=True)
    assert layer.forward_host(x_host, out=out) is out and torch.equal(out, got)
    if opts.get("bias") is None and ref.dtype == torch.float32:
        qn = quantize_int4_groupwise(w.cpu().numpy(), g)
        xn = x.float().cpu().numpy()
        check_against_oracle(got, xn, qn, g, dtype)
    with pytest.raises(ValueError, match="page-locked"):
        layer.forward_host(x.cpu())
    with pytest.raises(ValueError, match="page-locked"):
        layer.forward_host(x_host, out=torch.empty(ref.shape, dtype=ref.dtype))
    with pytest.raises(ValueError):
        layer.forward_host(x)


@pytest.mark.parametrize("shape", [(77, 300, 512, 32, torch.float16), (300, 1000, 2048, 128, torch.bfloat16),
                                   (2048, 700, 1024, 128, torch.bfloat16), (17, 2000, 4096, 128, torch.float16),
                                   (40, 64, 256, 64, torch.float16), (8, 100, 1024, 128, torch.bfloat16)])
def test_silu_gate_fusion_prefill_gemm(shape):
    """silu_gate on the tcgen05 GEMM (M > 16, or kernel="tcgen05"): tiles
    pair each feature's gate and up rows and the epilogue writes
    silu(gate) * up.  Equal to silu(gate) * up of two plain GEMM launches
    (the same sums; silu from expf vs torch's sigmoid in fp64: a few ulp),
    within the parity bar of the oracle's two products, through int4_linear,
    with bf16 output, and unchanged when a workspace is offered (the fused
    GEMM never splits)."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import int4_linear
    from openquant_b200 import _native as nat

    m, n, k, g, dtype = shape
    gen = torch.Generator(device="cuda").manual_seed(3 * n + k)
    w = torch.randn(2 * n, k, device="cuda", generator=gen).mul_(0.02).to(dtype)
    q = quantize_int4_groupwise(w, g)
    x = torch.randn(m, k, device="cuda", generator=gen).to(dtype)
    code = nat.OQ_F16 if dtype == torch.float16 else nat.OQ_BF16
    lib = nat.load()
    half = q.data.numel() // 2
    tc = nat.KERNELS["tcgen05"]

    def run(packed, scales, out_cols, kernel, cfg):
        y = torch.empty(m, out_cols, device="cuda")
        nat.check(lib.oq_int4_linear(nat.ptr(x), code, nat.ptr(packed), nat.ptr(scales), nat.ptr(y), m, out_cols, k,
                                     g, kernel, cfg, nat.stream_of(x.device)))
        return y

    gate = run(q.data[:half], q.scales[:n], n, tc, 0)
    up = run(q.data[half:], q.scales[n:], n, tc, 0)
    fused = run(q.data, q.scales, n, tc, nat.CONFIG_SILU_GATE)
    assert_no_device_error()
    ref = (gate.double() * torch.sigmoid(gate.double())) * up.double()
    err = (fused.double() - ref).abs()
    assert float((err - 2e-6 * ref.abs()).max()) <= 1e-6, float(err.max())
    if m > 16:
        assert torch.equal(run(q.data, q.scales, n, 0, nat.CONFIG_SILU_GATE), fused)
        assert torch.equal(int4_linear(x, q.data, q.scales, n, g, silu_gate=True), fused)
    assert torch.equal(int4_linear(x, q.data, q.scales, n, g, silu_gate=True, kernel="tcgen05"), fused)
    ws = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    y_ws = torch.empty(m, n, device="cuda")
    nat.check(lib.oq_int4_linear_ws(nat.ptr(x), code, nat.ptr(q.data), nat.ptr(q.scales), nat.ptr(y_ws), nat.OQ_F32,
                                    None, m, n, k, g, tc, nat.CONFIG_SILU_GATE, nat.ptr(ws), ws.numel(),
                                    nat.stream_of(x.device)))
    assert torch.equal(y_ws, fused)
    name = "f16" if dtype == torch.float16 else "bf16"
    data, scales = q.data.cpu().numpy(), q.scales.cpu().numpy()
    xf = x.float().cpu().numpy()
    g_ref = orc.int4_linear(xf, data[:half], scales[:n], n, g, x_dtype=name)
    u_ref = orc.int4_linear(xf, data[half:], scales[n:], n, g, x_dtype=name)
    silu = g_ref / (1.0 + np.exp(-g_ref))
    ref_o = silu * u_ref
    err_o = fused.double().cpu().numpy() - ref_o
    assert (np.abs(err_o) <= MAX_ABS * (1.1 * np.abs(u_ref) + np.abs(silu)) + 1e-6).all()
    assert np.linalg.norm(err_o) / np.linalg.norm(ref_o) <= 2 * REL_L2
    yb = int4_linear(x, q.data, q.scales, n, g, silu_gate=True, kernel="tcgen05", out_dtype=torch.bfloat16)
    assert torch.equal(yb, fused.to(torch.bfloat16))
    with pytest.raises(ValueError):
        int4_linear(x, q.data, q.scales, n, g, silu_gate=True, kernel="simt")


def test_forward_host_plan_replays_new_inputs():
    """A captured host call (Int4Linear's plan for one (x, out) pair) reads x
    at every run: new contents of the same page-locked x give the new result;
    more (x, out) pairs than the plan cache holds still compute correctly;
    and the uncaptured C entry point oq_int4_linear_host agrees bit for bit."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.triton_int4 import Int4Linear
    from openquant_b200.triton_int4 import _PLANS
    from openquant_b200 import _native as nat

    m, n, k, g = 1, 4096, 4096, 128
    gen = torch.Generator(device="cuda").manual_seed(11)
    q = quantize_int4_groupwise(torch.randn(n, k, device="cuda", generator=gen).mul_(0.02), g)
    layer = Int4Linear(q.data, q.scales, n, g, static_weights=True)
    x_host = torch.empty(m, k, dtype=torch.float16, pin_memory=True)
    out = torch.empty(m, n, pin_memory=True)
    for i in range(3):
        x = torch.randn(m, k, device="cuda", generator=gen).half()
        x_host.copy_(x.cpu())
        assert layer.forward_host(x_host, out=out) is out
        assert torch.equal(out, layer(x).cpu()), i
    pairs = [(torch.randn(m, k, generator=torch.Generator().manual_seed(i)).half().pin_memory(),
              torch.empty(m, n, pin_memory=True)) for i in range(_PLANS + 3)]
    for xh, yh in pairs + pairs[:2]:
        assert torch.equal(layer.forward_host(xh, out=yh), layer(xh.cuda()).cpu())
    assert len(layer._plans) <= _PLANS
    lib = nat.load()
    xh, yh = pairs[0]
    y2 = torch.empty(m, n, pin_memory=True)
    stage = torch.empty(m, k, dtype=torch.float16, device="cuda")
    st = lib.oq_int4_linear_host(xh.data_ptr(), nat.OQ_F16, q.data.data_ptr(), q.scales.data_ptr(), y2.data_ptr(),
                                 nat.OQ_F32, None, m, n, k, g, 0, nat.CONFIG_STATIC_WEIGHTS, stage.data_ptr(),
                                 nat.stream_of(torch.device("cuda")))
    assert st == 0, nat.last_error()
    assert torch.equal(y2, yh)
    assert lib.oq_int4_linear_host(xh.data_ptr(), nat.OQ_F16, q.data.data_ptr(), q.scales.data_ptr(),
                                   torch.empty(m, n).data_ptr(), nat.OQ_F32, None, m, n, k, g, 0, 0,
                                   stage.data_ptr(), nat.stream_of(torch.device("cuda"))) == nat.OQ_ERR_INVALID
    assert "page-locked" in nat.last_error()


@pytest.mark.parametrize("case", [(300, 1000, 2048, 128, torch.bfloat16),   # 16 tiles, each cut over ~9 SMs
                                  (77, 700, 1024, 64, torch.float16),
                                  (300, 19456, 2048, 128, torch.bfloat16),  # 304 tiles: 2 rounds + 8 split
                                  (1100, 2000, 512, 128, torch.bfloat16)],  # wide tiles, split
                         ids=lambda c: f"m{c[0]}_n{c[1]}_k{c[2]}_g{c[3]}")
def test_gemm_even_split_against_unsplit_and_oracle(case):
    """The tcgen05 GEMM with a workspace splits the tiles' k-blocks evenly
    over the SMs (stream-K) and adds the pieces in k order: deterministic
    (two calls bit-equal), the unsplit kernel's result up to fp32 summation
    order, the parity bar against the oracle, the fused epilogue (bias,
    bf16 output) applied once to the added pieces; and with a workspace one
    byte short it runs the unsplit kernel, bit for bit."""
    from openquant_b200 import _native as nat

    m, n, k, g, dtype = case
    lib = nat.load()
    x, q, xt = make_case(m, n, k, g, dtype, seed=m + k, w_sigma=0.02)
    p, s = torch.from_numpy(q.data).cuda(), torch.from_numpy(q.scales).cuda()
    code = nat.OQ_F16 if dtype == torch.float16 else nat.OQ_BF16
    tc = nat.KERNELS["tcgen05"]
    ws_bytes = lib.oq_int4_linear_workspace_bytes(m, n, k, g, tc, 0)
    assert ws_bytes > 0, "this shape should take the split"
    st = nat.stream_of(xt.device)

    def run(ws_size, ydt=torch.float32, bias=None):
        y = torch.full((m, n), float("nan"), device="cuda").to(ydt)
        ws = torch.empty(max(ws_size, 16), dtype=torch.uint8, device="cuda")
        nat.check(lib.oq_int4_linear_ws(nat.ptr(xt), code, nat.ptr(p), nat.ptr(s), nat.ptr(y),
                                        {torch.float32: nat.OQ_F32, torch.bfloat16: nat.OQ_BF16}[ydt],
                                        nat.ptr(bias) if bias is not None else None, m, n, k, g, tc, 0,
                                        nat.ptr(ws), ws_size, st))
        return y

    y1, y2 = run(ws_bytes), run(ws_bytes)
    assert torch.equal(y1, y2)
    plain = torch.empty(m, n, device="cuda")
    nat.check(lib.oq_int4_linear(nat.ptr(xt), code, nat.ptr(p), nat.ptr(s), nat.ptr(plain), m, n, k, g, tc, 0, st))
    assert ((y1.double() - plain.double()).norm() / plain.double().norm()).item() < 1e-5
    check_against_oracle(y1, x, q, g, dtype)
    bias = torch.randn(n, device="cuda")
    assert torch.equal(run(ws_bytes, torch.bfloat16, bias), (y1 + bias).to(torch.bfloat16))
    assert torch.equal(run(ws_bytes - 1), plain)


@pytest.mark.parametrize("shape", [(1, 4096, 4096, 128), (16, 12288, 4096, 128), (4, 4096, 11008, 128),
                                   (5, 300, 1000, 128)],
                         ids=lambda s: "m%d_n%d_k%d_g%d" % s)
def test_fp16_scales_vs_oracle(shape):
    """int4_linear(..., fp16_scales=True): one fp16 scale per group, on the
    decode GEMV (the pair GEMV where it takes the shape, else the TMA GEMV).
    The oracle is the reference's arithmetic with those scales widened to fp32
    (W = round_fp16(q * s)); same parity bar."""
    from openquant.triton_int4 import int4_linear

    m, n, k, g = shape
    x, q, xt = make_case(m, n, k, g, torch.float16, seed=n + k, w_sigma=0.02)
    s16 = q.scales.astype(np.float16)
    p = torch.from_numpy(q.data).cuda()
    y = int4_linear(xt, p, torch.from_numpy(s16).cuda(), n, g, fp16_scales=True)
    ref = orc.int4_linear(x, q.data, s16.astype(np.float32), n, g, x_dtype="f16")
    err = y.cpu().double().numpy() - ref
    assert np.linalg.norm(err) / np.linalg.norm(ref) <= REL_L2
    assert np.abs(err).max() <= MAX_ABS
    # the fp32-scale call with the same scales widened: the same sums up to the
    # launch shape's fp32 summation order (the tuned table may pick another)
    y32 = int4_linear(xt, p, torch.from_numpy(s16.astype(np.float32)).cuda(), n, g)
    assert ((y.double() - y32.double()).norm() / y32.double().norm()).item() < 1e-4
    with pytest.raises(ValueError):  # the reference's contract stays: fp32 scales without the flag
        int4_linear(xt, p, torch.from_numpy(s16).cuda(), n, g)
    with pytest.raises(ValueError):
        int4_linear(xt.to(torch.bfloat16), p, torch.from_numpy(s16).cuda(), n, g, fp16_scales=True)
