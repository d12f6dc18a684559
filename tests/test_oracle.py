"""Pins the CPU oracle to the golden vectors recorded from the reference.

Every packed byte, scale and dequantized value the reference produced must
come out of the oracle bit for bit; the full-size cases are compared by
SHA-256 digest.  CPU only.
"""
import numpy as np
import pytest

import cases
import oq_oracle as orc
from conftest import assert_matches_golden, sha256

ROW = cases.rowwise_cases()
GROUP = cases.group_cases()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("name", sorted(ROW))
def test_rowwise_oracle_matches_reference(golden, name, bits):
    w = ROW[name]
    data, scales = orc.quantize(w, bits)
    key = f"row{bits}/{name}"
    assert_matches_golden(golden, key + "/data", data)
    assert_matches_golden(golden, key + "/scales", scales)
    with np.errstate(all="ignore"):
        deq = orc.dequantize(data, scales, bits, w.shape)
    assert_matches_golden(golden, key + "/dequant", deq)
    assert_matches_golden(golden, key + "/decode_gpu", deq)


@pytest.mark.parametrize("name", sorted(GROUP))
def test_group_oracle_matches_reference(golden, name):
    w, g = GROUP[name]
    data, scales = orc.quantize_int4_groupwise(w, g)
    key = f"group/{name}"
    assert_matches_golden(golden, key + "/data", data)
    assert_matches_golden(golden, key + "/scales", scales)
    deq = np.ascontiguousarray(orc.dequantize_int4_groupwise(data, scales, w.shape, g))
    assert_matches_golden(golden, key + "/dequant", deq)
    assert_matches_golden(golden, key + "/restore_torch", deq)


@pytest.mark.parametrize("name", sorted(cases.hashed_cases()))
def test_full_size_oracle_matches_reference(golden, name):
    _, meta = golden
    entry = meta["cases"][name]
    (kind, param), recipe = cases.hashed_cases()[name]
    w = recipe()
    if kind == "rowwise":
        data, scales = orc.quantize(w, param)
    else:
        data, scales = orc.quantize_int4_groupwise(w, param)
    assert data.nbytes == entry["data_nbytes"]
    assert list(scales.shape) == entry["scales_shape"]
    assert sha256(data) == entry["data_sha256"]
    assert sha256(scales) == entry["scales_sha256"]


def test_oracle_validation_errors():
    with pytest.raises(ValueError):
        orc.quantize(np.ones((2, 2)), bits=3)
    with pytest.raises(ValueError):
        orc.quantize(np.ones(10), bits=8)
    for g in (0, 1, 3):
        with pytest.raises(ValueError):
            orc.quantize_int4_groupwise(np.ones((2, 8)), g)
    with pytest.raises(ValueError):
        orc.quantize_int4_groupwise(np.ones(8))
    with pytest.raises(ValueError):
        orc.quantize_int4_groupwise(np.zeros((0, 8)))
    with pytest.raises(ValueError):
        orc.quantize_int4_groupwise(np.array([[1.0, np.nan]]))


def test_round_to_dtype_bf16_matches_torch():
    import torch

    a = np.random.default_rng(0).normal(0, 3, 10000).astype(np.float32)
    a[:4] = [np.float32(1.00390625), np.float32(1.01171875), np.float32(-2.0078125), 3.0e38]
    ref = torch.from_numpy(a).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(orc.round_to_dtype(a, "bf16"), ref)
    ref16 = torch.from_numpy(a).to(torch.float16).float().numpy()
    np.testing.assert_array_equal(orc.round_to_dtype(a, "f16"), ref16)
