"""CLI verbs end to end on the GPU; mirrors the reference's tests/test_report.py."""
import json

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")


@pytest.mark.parametrize("rows,cols,group", [(3, 5, 4), (4, 7, 16)])
def test_report_shapes(rows, cols, group):
    from openquant.report import make_cpu_report

    result = make_cpu_report(rows, cols, seed=7, group_size=group)
    assert result["weights"]["shape"] == [rows, cols]
    for name in ("FP32", "INT8", "INT4", f"INT4_GROUP_{group}"):
        assert result["formats"][name]["storage_bytes"] > 0


def test_report_reproducibility():
    from openquant.report import make_cpu_report

    assert make_cpu_report(16, 32, seed=42)["formats"] == make_cpu_report(16, 32, seed=42)["formats"]


def test_report_matches_oracle_errors():
    import numpy as np

    import oq_oracle as orc
    from openquant.report import make_cpu_report

    rep = make_cpu_report(64, 96, seed=3, group_size=32)
    w = np.random.default_rng(3).normal(0, 0.2, (64, 96)).astype(np.float32)
    d, s = orc.quantize_int4_groupwise(w, 32)
    r = orc.dequantize_int4_groupwise(d, s, w.shape, 32)
    err = round(100 * float(np.linalg.norm(w - r) / np.linalg.norm(w)), 6)
    assert rep["formats"]["INT4_GROUP_32"]["relative_weight_error_pct"] == err


def test_cli_report_json(tmp_path):
    from openquant.cli import main

    out = tmp_path / "report.json"
    assert main(["report", "--rows", "8", "--cols", "16", "--group-size", "8", "--output", str(out)]) == 0
    data = json.loads(out.read_text(encoding="utf-8"))
    assert data["schema_version"] == 1 and "INT4_GROUP_8" in data["formats"]


def test_cli_cpu_and_gpu(capsys):
    from openquant.cli import main

    assert main(["cpu", "--rows", "32", "--cols", "32"]) == 0
    out = capsys.readouterr().out
    assert "INT8" in out and "INT4" in out and "Relative weight error" in out
    assert main(["gpu"]) == 0
    out = capsys.readouterr().out
    assert "Fused B200 INT4" in out and "TFLOP/s" in out


def test_cli_tune_quick(tmp_path):
    from openquant.cli import main
    from openquant_b200 import tile_table

    out = tmp_path / "table.json"
    assert main(["tune", "--quick", "--output", str(out)]) == 0
    data = json.loads(out.read_text())
    assert len(data["entries"]) == 1 and data["entries"][0]["key"] == [128, 2048, 2048, 32]
    tile_table.reset()


def test_gpu_report_schema_2(tmp_path):
    from openquant.cli import main

    out = tmp_path / "gpu.json"
    assert main(["report", "--gpu", "--rows", "512", "--cols", "1024", "--group-size", "128", "--batch", "4",
                 "--output", str(out)]) == 0
    data = json.loads(out.read_text(encoding="utf-8"))
    assert data["schema_version"] == 2 and data["weights"]["shape"] == [512, 1024]
    fm = data["gpu"]["formats"]
    assert set(fm) == {"INT8", "INT4", "INT4_GROUP_128"}
    assert {"quantize_fp16", "dequantize", "w8a8_linear"} <= set(fm["INT8"])
    assert "int4_linear" in fm["INT4_GROUP_128"]
    for kernels in fm.values():
        for k in kernels.values():
            assert k["time_us"] > 0 and k["GB_per_s"] > 0
    # schema-1 content is unchanged
    assert data["formats"]["INT4_GROUP_128"]["storage_bytes"] == 512 * 1024 // 2 + 512 * 8 * 4
