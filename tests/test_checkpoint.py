"""On-disk packed-weight format: round trips on the host and malformed files."""
import numpy as np
import pytest

import oq_oracle as orc
from openquant_b200.checkpoint import ALIGN, MAGIC, load, save
from openquant_b200.groupwise import Groupwise4
from openquant_b200.quantization import QuantizedWeights


def _weights():
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (40, 300)).astype(np.float32)
    d, s = orc.quantize_int4_groupwise(w, 32)
    d8, s8 = orc.quantize(w, 8)
    d4, s4 = orc.quantize(w[:7, :13], 4)
    return {
        "layers.0.mlp": Groupwise4(data=d, scales=s, shape=w.shape, group_size=32),
        "layers.0.attn": QuantizedWeights(data=d8, scales=s8, bits=8, shape=w.shape),
        "odd": QuantizedWeights(data=d4, scales=s4, bits=4, shape=(7, 13)),
    }


def test_round_trip_on_the_host(tmp_path):
    src = _weights()
    path = tmp_path / "w.oqb"
    save(path, src)
    got = load(path, device="cpu")
    assert set(got) == set(src)
    for name, obj in src.items():
        g = got[name]
        assert type(g) is type(obj) and tuple(g.shape) == tuple(obj.shape)
        np.testing.assert_array_equal(g.data, obj.data)
        np.testing.assert_array_equal(g.scales.view(np.uint32), np.asarray(obj.scales).view(np.uint32))
    assert got["layers.0.mlp"].group_size == 32 and got["odd"].bits == 4
    with open(path, "rb") as f:
        assert f.read(8) == MAGIC


def test_arrays_are_aligned_and_file_is_tight(tmp_path):
    path = tmp_path / "w.oqb"
    save(path, _weights())
    import json
    import struct

    with open(path, "rb") as f:
        f.read(8)
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
    metas = [a for e in header["entries"].values() for a in e["arrays"].values()]
    assert all(m["offset"] % ALIGN == 0 for m in metas)
    assert path.stat().st_size == max(m["offset"] + m["nbytes"] for m in metas)


def test_malformed_files_raise(tmp_path):
    path = tmp_path / "w.oqb"
    save(path, _weights())
    raw = path.read_bytes()
    bad = tmp_path / "bad.oqb"
    bad.write_bytes(b"NOTACKPT" + raw[8:])
    with pytest.raises(ValueError, match="magic"):
        load(bad, device="cpu")
    bad.write_bytes(raw[:len(raw) - 100])
    with pytest.raises(ValueError, match="truncated"):
        load(bad, device="cpu")
    with pytest.raises(TypeError):
        save(tmp_path / "x.oqb", {"w": np.zeros(4)})
