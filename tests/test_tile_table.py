"""The tuned kernel table and the tuner's candidate rules (CPU only: no
kernel runs here)."""
import json

from openquant_b200 import _native as nat
from openquant_b200 import autotune, tile_table


def test_candidates_include_the_automatic_choice_and_keep_the_rounding():
    for m in (1, 4, 16, 17, 64, 128, 2048):
        cands = autotune.candidates(m)
        assert cands[0] == ("auto", 0, 0)
        gemv = [cfg for name, kern, cfg in cands if kern == nat.KERNELS["gemv"]]
        # a table entry changes the launch shape, never the rounding: the
        # exact-rounding flag is set exactly where the library's default is
        # exact rounding (M > 16)
        assert all(bool(cfg & nat.CONFIG_EXACT_ROUNDING) == (m > 16) for cfg in gemv)
        assert all((cfg & 15) != 11 for cfg in gemv)  # 11 is not a launch shape
    assert not [c for c in autotune.candidates(128) if c[1] == nat.KERNELS["gemv"]]


def test_committed_table_is_well_formed():
    with open(tile_table.TABLE_PATH) as f:
        data = json.load(f)
    assert data["entries"]
    for e in data["entries"]:
        bucket, n, k, g = e["key"]
        assert bucket == tile_table.m_bucket(bucket) and n > 0 and k > 0 and g > 0
        assert e["kernel"] in nat.KERNELS.values()
        if e["kernel"] == nat.KERNELS["gemv"]:
            assert 1 <= (e["split_k"] & 15) <= 13 and (e["split_k"] & 15) != 11
        assert e["us"] > 0


def test_lookup_uses_the_batch_bucket_and_defaults_to_auto():
    tile_table.reset()
    table = tile_table.load_table()
    for (bucket, n, k, g), choice in table.items():
        # every M of the bucket maps to the entry
        lo = bucket // 2 + 1 if bucket > 1 else 1
        for m in {lo, bucket}:
            assert tile_table.lookup(m, n, k, g) == choice
    assert tile_table.lookup(3, 12345, 678, 64) == (0, 0)
    assert [tile_table.m_bucket(m) for m in (1, 2, 3, 4, 5, 16, 17, 2048)] == [1, 2, 4, 4, 8, 16, 32, 2048]
