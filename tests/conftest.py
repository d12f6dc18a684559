import hashlib
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, os.path.join(ROOT, "oracle"), GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device with compute capability 10.x (B200)")


def sha256(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="session")
def golden():
    with np.load(os.path.join(GOLDEN, "golden.npz")) as z:
        arrays = {k: z[k] for k in z.files}
    with open(os.path.join(GOLDEN, "golden_hashes.json")) as f:
        meta = json.load(f)
    return arrays, meta


def golden_array(golden, key):
    """The stored array, or None plus its digest when only a digest is kept."""
    arrays, meta = golden
    if key in arrays:
        return arrays[key], None
    return None, meta["arrays"][key]


def assert_matches_golden(golden, key, actual, exact=True, atol=0.0):
    expected, digest = golden_array(golden, key)
    actual = np.ascontiguousarray(actual)
    if expected is None:
        assert sha256(actual.astype(np.float32)) == digest, key
        return
    assert actual.shape == expected.shape or actual.size == expected.size, (key, actual.shape, expected.shape)
    actual = actual.reshape(expected.shape)
    if exact:
        if expected.dtype.kind == "f":
            assert_float_bits_equal(actual, expected, key)
        else:
            np.testing.assert_array_equal(actual, expected, err_msg=key)
    else:
        np.testing.assert_allclose(actual, expected, rtol=0, atol=atol, err_msg=key)


def assert_float_bits_equal(actual, expected, msg=""):
    """Bit-for-bit equality of float arrays (so -0.0 != +0.0), except that a
    NaN only has to meet a NaN: x86 and NVIDIA GPUs write different NaN
    payloads (0x7FC00000 / 0xFFC00000 vs 0x7FFFFFFF), which carry no value."""
    actual = np.asarray(actual, dtype=np.float32)
    expected = np.asarray(expected, dtype=np.float32)
    assert actual.shape == expected.shape, (msg, actual.shape, expected.shape)
    nan_a, nan_e = np.isnan(actual), np.isnan(expected)
    np.testing.assert_array_equal(nan_a, nan_e, err_msg=f"{msg}: NaN positions")
    keep = ~nan_e
    np.testing.assert_array_equal(actual.view(np.uint32)[keep], expected.view(np.uint32)[keep], err_msg=msg)
