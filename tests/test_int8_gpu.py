"""W8A8 path: per-token INT8 activations (the reference's quantize(bits=8)
format, one row per token) times per-row INT8 weights on the tcgen05 tensor
cores, against the oracle.  The integer sums are exact, so each output may
differ from the float64 oracle only by the three fp32 roundings of the
epilogue (int32 -> fp32, times sw, times sx): |y - ref| <= 4e-7 |ref|.
"""
import numpy as np
import pytest
import torch

import oq_oracle as orc

pytestmark = pytest.mark.gpu
RTOL = 4e-7


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    from openquant_b200 import build

    build.build()


def _check(y, ref):
    got = y.cpu().numpy().astype(np.float64)
    assert got.shape == ref.shape
    err = np.abs(got - ref)
    bound = RTOL * np.abs(ref)
    bad = np.flatnonzero(err > bound)
    assert bad.size == 0, f"{bad.size} outputs off, worst rel {float((err / np.maximum(np.abs(ref), 1e-30)).max()):.3g}"


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_activation_quantization_is_the_reference_format(dtype):
    from openquant_b200.int8_linear import quantize_activations

    rng = np.random.default_rng(1)
    x = torch.from_numpy(rng.normal(size=(37, 1040)).astype(np.float32)).to(dtype)
    qx, sx = quantize_activations(x.cuda())
    d, s = orc.quantize(x.float().numpy(), 8)
    np.testing.assert_array_equal(qx.cpu().numpy(), d)
    np.testing.assert_array_equal(sx.cpu().numpy().view(np.uint32), s.reshape(-1).view(np.uint32))


@pytest.mark.parametrize("m,n,k", [(1, 16, 16), (3, 130, 48), (300, 1000, 4096), (257, 129, 8208), (64, 28672, 128),
                                   (2048, 8192, 256)])
def test_int8_gemm_vs_oracle(m, n, k):
    # (2048, 8192, 256): 512 tiles, so every CTA cycles both TMEM accumulators.
    from openquant_b200.int8_linear import int8_matmul

    rng = np.random.default_rng(m + n + k)
    qx = rng.integers(-127, 128, (m, k), dtype=np.int8)
    qw = rng.integers(-127, 128, (n, k), dtype=np.int8)
    sx = rng.uniform(1e-3, 1e-1, m).astype(np.float32)
    sw = rng.uniform(1e-3, 1e-1, n).astype(np.float32)
    y = int8_matmul(*(torch.from_numpy(a).cuda() for a in (qx, sx, qw, sw)))
    _check(y, orc.int8_matmul(qx, sx, qw, sw))
    # a second call into the same output (persistent grid, reused TMEM)
    y2 = int8_matmul(*(torch.from_numpy(a).cuda() for a in (qx, sx, qw, sw)), out=y)
    _check(y2, orc.int8_matmul(qx, sx, qw, sw))


def test_int8_linear_end_to_end():
    from openquant.quantization import quantize
    from openquant_b200.int8_linear import int8_linear, quantize_activations

    rng = np.random.default_rng(7)
    w = rng.normal(0, 0.02, (512, 2048)).astype(np.float32)
    x = rng.normal(size=(33, 2048)).astype(np.float32)
    qw = quantize(torch.from_numpy(w).cuda(), 8)
    xt = torch.from_numpy(x).cuda().to(torch.bfloat16)
    y = int8_linear(xt, qw)
    qx, sx = quantize_activations(xt)
    _check(y, orc.int8_matmul(qx.cpu().numpy(), sx.cpu().numpy(), qw.data.cpu().numpy(), qw.scales.cpu().numpy()))
    # and close to the unquantized product (INT8 on both sides: ~1 % error)
    ref = xt.double().cpu().numpy() @ w.T.astype(np.float64)
    rel = np.linalg.norm(y.cpu().numpy() - ref) / np.linalg.norm(ref)
    assert rel < 0.02, rel


def test_int8_gemm_argument_errors():
    from openquant_b200.int8_linear import int8_matmul

    qx = torch.zeros((4, 24), dtype=torch.int8, device="cuda")
    qw = torch.zeros((8, 24), dtype=torch.int8, device="cuda")
    s4, s8 = torch.ones(4, device="cuda"), torch.ones(8, device="cuda")
    with pytest.raises(ValueError, match="multiple of 16"):
        int8_matmul(qx, s4, qw, s8)
    with pytest.raises(ValueError, match="scales"):
        int8_matmul(torch.zeros((4, 32), dtype=torch.int8, device="cuda"), s8,
                    torch.zeros((8, 32), dtype=torch.int8, device="cuda"), s8)
