"""Streaming packed weights from disk into HBM (pinned, double-buffered)."""
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _device():
    if not torch.cuda.is_available():
        pytest.skip("CUDA GPU required")


def test_stream_to_gpu_round_trip(tmp_path):
    from openquant.groupwise import quantize_int4_groupwise
    from openquant.quantization import quantize
    from openquant.triton_int4 import int4_linear
    from openquant_b200.checkpoint import load, save

    gen = torch.Generator(device="cuda").manual_seed(5)
    layers = {}
    for i in range(3):
        w = torch.randn(1536, 4096, device="cuda", generator=gen).mul_(0.02).half()
        layers[f"l{i}.g"] = quantize_int4_groupwise(w, 128)
        layers[f"l{i}.q"] = quantize(w[:100], 8)
    path = tmp_path / "model.oqb"
    save(path, layers)
    t0 = time.perf_counter()
    got = load(path, device="cuda", chunk_bytes=1 << 20)  # 1 MB chunks: chunks straddle arrays
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    print(f"loaded {path.stat().st_size / 1e6:.1f} MB in {dt * 1e3:.1f} ms")
    for name, obj in layers.items():
        g = got[name]
        assert g.data.is_cuda and g.scales.is_cuda
        assert torch.equal(g.data, obj.data)
        assert torch.equal(g.scales.view(torch.int32), obj.scales.view(torch.int32))
    x = torch.randn(1, 4096, device="cuda", generator=gen).half()
    y0 = int4_linear(x, layers["l1.g"].data, layers["l1.g"].scales, 1536, 128)
    y1 = int4_linear(x, got["l1.g"].data, got["l1.g"].scales, 1536, 128)
    assert torch.equal(y0, y1)
