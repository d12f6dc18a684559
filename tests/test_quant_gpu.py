"""Quantize / dequantize kernels vs the reference's golden vectors and the
oracle, bit for bit.  Mirrors tests/test_quantization.py,
tests/test_groupwise.py and tests/test_gpu_decode.py of the reference, run
through the CUDA path.
"""
import numpy as np
import pytest
import torch

import cases
import oq_oracle as orc
from conftest import assert_matches_golden, sha256

pytestmark = pytest.mark.gpu

ROW = cases.rowwise_cases()
GROUP = cases.group_cases()


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")
    from openquant_b200 import build

    build.build()


def _np(t):
    return t.detach().cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)


# ----------------------------------------------------------- per-row --


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("name", sorted(ROW))
def test_rowwise_host_path_matches_reference(golden, name, bits):
    from openquant.quantization import dequantize, quantize
    from openquant.gpu_benchmark import decode_gpu

    w = ROW[name]
    q = quantize(w, bits)
    assert isinstance(q.data, np.ndarray) and q.shape == w.shape and q.bits == bits
    key = f"row{bits}/{name}"
    assert_matches_golden(golden, key + "/data", q.data)
    assert_matches_golden(golden, key + "/scales", q.scales)
    assert q.scales.shape == (w.shape[0], 1)
    assert_matches_golden(golden, key + "/dequant", dequantize(q))
    dec = decode_gpu(torch.from_numpy(q.data), torch.from_numpy(q.scales), bits, w.shape)
    assert dec.device.type == "cpu"
    assert_matches_golden(golden, key + "/decode_gpu", dec.numpy())


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64, torch.bfloat16])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("name", ["n02_9x31_bf16", "n002_64x1000", "edge_nonfinite", "ties_int4", "n002_33x65"])
def test_rowwise_device_path_matches_reference(golden, name, bits, dtype):
    from openquant.quantization import dequantize, quantize

    w = ROW[name]
    if dtype == torch.bfloat16 and not np.array_equal(cases.bf16_exact(w), w, equal_nan=True):
        pytest.skip("values not representable in bf16")
    wd = torch.from_numpy(w).to(dtype).cuda()
    q = quantize(wd, bits)
    assert q.data.is_cuda and q.scales.is_cuda
    key = f"row{bits}/{name}"
    assert_matches_golden(golden, key + "/data", _np(q.data))
    assert_matches_golden(golden, key + "/scales", _np(q.scales))
    assert_matches_golden(golden, key + "/dequant", _np(dequantize(q)))


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("shape", [(1, 1), (1, 2), (2, 1), (3, 3), (7, 5), (5, 8), (3, 17), (9, 1031), (64, 4096)])
def test_rowwise_ragged_shapes_vs_oracle(bits, shape):
    from openquant.quantization import dequantize, quantize

    rng = np.random.default_rng(sum(shape) * bits)
    w = rng.normal(0, 0.05, shape).astype(np.float32)
    w[0, 0] = 0.0
    data, scales = orc.quantize(w, bits)
    q = quantize(w, bits)
    np.testing.assert_array_equal(q.data, data)
    np.testing.assert_array_equal(q.scales.view(np.uint32), scales.view(np.uint32))
    np.testing.assert_array_equal(dequantize(q), orc.dequantize(data, scales, bits, shape))


def test_rowwise_zero_rows_and_storage():
    from openquant.quantization import dequantize, quantize

    w = np.array([[0, 0, 0], [1, -1, 0.5], [0, -0.5, 1]], np.float32)
    for bits in (4, 8):
        r = dequantize(quantize(w, bits))
        assert r.shape == (3, 3) and np.all(np.isfinite(r)) and np.all(r[0] == 0)
        ones = quantize(np.ones((17, 19), np.float32), bits)
        assert ones.data.nbytes == (17 * 19 if bits == 8 else (17 * 19 + 1) // 2)


@pytest.mark.parametrize("bits,limit", [(8, 0.02), (4, 0.20)])
def test_reconstruction_error(bits, limit):
    from openquant.quantization import dequantize, quantize

    w = np.random.default_rng(42).normal(size=(128, 256)).astype(np.float32)
    r = dequantize(quantize(w, bits))
    assert np.linalg.norm(w - r) / np.linalg.norm(w) < limit


# --------------------------------------------------------- groupwise --


@pytest.mark.parametrize("name", sorted(GROUP))
def test_group_host_path_matches_reference(golden, name):
    from openquant.groupwise import dequantize_int4_groupwise, quantize_int4_groupwise
    from openquant.group_benchmark import restore_groupwise_torch

    w, g = GROUP[name]
    q = quantize_int4_groupwise(w, g)
    assert q.shape == w.shape and q.group_size == g
    key = f"group/{name}"
    assert_matches_golden(golden, key + "/data", q.data)
    assert_matches_golden(golden, key + "/scales", q.scales)
    assert_matches_golden(golden, key + "/dequant", dequantize_int4_groupwise(q))
    rest = restore_groupwise_torch(torch.from_numpy(q.data), torch.from_numpy(q.scales), w.shape, g)
    assert rest.device.type == "cpu"
    assert_matches_golden(golden, key + "/restore_torch", rest.numpy())


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("name", ["n002_16x512_g8_bf16", "n002_32x4096_g128_bf16", "n1_3x67_g16", "n1_6x40_g6",
                                  "n002_24x96_g256", "ties_3x13_g14"])
def test_group_device_path_matches_reference(golden, name, dtype):
    from openquant.groupwise import dequantize_int4_groupwise, quantize_int4_groupwise

    w, g = GROUP[name]
    wt = torch.from_numpy(w).to(dtype)
    if not np.array_equal(wt.double().numpy(), w.astype(np.float64)):
        pytest.skip("values not representable in this dtype")
    q = quantize_int4_groupwise(wt.cuda(), g)
    assert q.data.is_cuda
    key = f"group/{name}"
    assert_matches_golden(golden, key + "/data", _np(q.data))
    assert_matches_golden(golden, key + "/scales", _np(q.scales))
    assert_matches_golden(golden, key + "/dequant", _np(dequantize_int4_groupwise(q)))


@pytest.mark.parametrize("g", [2, 4, 6, 8, 16, 32, 64, 128, 256, 512, 10])
@pytest.mark.parametrize("shape", [(1, 1), (3, 7), (5, 64), (2, 129), (17, 520)])
def test_group_ragged_shapes_vs_oracle(shape, g):
    from openquant.groupwise import dequantize_int4_groupwise, quantize_int4_groupwise

    rng = np.random.default_rng(shape[0] * 1000 + shape[1] + g)
    w = rng.normal(0, 0.05, shape).astype(np.float32)
    data, scales = orc.quantize_int4_groupwise(w, g)
    q = quantize_int4_groupwise(w, g)
    np.testing.assert_array_equal(q.data, data)
    np.testing.assert_array_equal(q.scales.view(np.uint32), scales.view(np.uint32))
    np.testing.assert_array_equal(dequantize_int4_groupwise(q), orc.dequantize_int4_groupwise(data, scales, shape, g))


def test_group_zero_weights_and_errors():
    from openquant.groupwise import dequantize_int4_groupwise, quantize_int4_groupwise

    q = quantize_int4_groupwise(np.zeros((2, 35), np.float32))
    assert np.all(dequantize_int4_groupwise(q) == 0)
    for bad in (np.nan, np.inf, -np.inf):
        w = np.ones((4, 70), np.float32)
        w[3, 69] = bad
        with pytest.raises(ValueError, match="finite"):
            quantize_int4_groupwise(w, 32)
        with pytest.raises(ValueError, match="finite"):
            quantize_int4_groupwise(torch.from_numpy(w).cuda(), 32)


# -------------------------------------------------- full-size digests --


@pytest.mark.parametrize("name", sorted(cases.hashed_cases()))
def test_full_size_cases_match_reference_digest(golden, name):
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.quantization import quantize

    entry = golden[1]["cases"][name]
    (kind, param), recipe = cases.hashed_cases()[name]
    w = torch.from_numpy(recipe()).cuda()
    q = quantize(w, param) if kind == "rowwise" else quantize_int4_groupwise(w, param)
    assert sha256(_np(q.data)) == entry["data_sha256"], name
    assert sha256(_np(q.scales)) == entry["scales_sha256"], name


def test_bulk_bf16_layer_sampled_rows_bit_exact():
    """A 70B-sized bf16 matrix (8192 x 28672) with 0.1 % outliers at 10
    sigma: quantize on the GPU, compare sampled rows with the oracle."""
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.quantization import quantize

    n, k = 8192, 28672
    gen = torch.Generator(device="cuda").manual_seed(1234)
    w = torch.randn(n, k, device="cuda", generator=gen, dtype=torch.float32).mul_(0.02)
    idx = torch.randint(0, n * k, (n * k // 1000,), device="cuda", generator=gen)
    w.view(-1)[idx] = 0.2 * torch.sign(torch.randn(idx.numel(), device="cuda", generator=gen))
    w = w.to(torch.bfloat16)
    rows = np.array([0, 1, 77, 4095, 8191])
    sample = w[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    q8 = quantize(w, 8)
    d, s = orc.quantize(sample, 8)
    np.testing.assert_array_equal(q8.data[torch.from_numpy(rows).cuda()].cpu().numpy(), d)
    np.testing.assert_array_equal(q8.scales[torch.from_numpy(rows).cuda()].cpu().numpy(), s)
    del q8
    for g in (32, 64, 128):
        qg = quantize_int4_groupwise(w, g)
        d, s = orc.quantize_int4_groupwise(sample, g)
        packed = qg.data.view(n, k // 2)[torch.from_numpy(rows).cuda()].cpu().numpy().reshape(-1)
        np.testing.assert_array_equal(packed, d)
        np.testing.assert_array_equal(qg.scales[torch.from_numpy(rows).cuda()].cpu().numpy(), s)
        del qg
