"""bench.py's CPU sample (the reported CPU baseline and the reference arm) on a small grid:
the dynamic path (zone statistics, shape choice, block selection) and the uniform path
(3D-chunk order, chunk selection) both run to a measured sample on the host cores."""
import importlib
import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture()
def bench():
    sys.path.insert(0, ROOT)
    import bench as b
    b = importlib.reload(b)  # fresh CONFIG for every case
    yield b


@pytest.mark.parametrize("path", ["dynamic", "uniform"])
def test_cpu_sample_runs(bench, path):
    bench.CONFIG.update(bench.CONFIGS["720p"])
    if path == "uniform":
        bench.CONFIG.update(bench.UNIFORM, method=None)
    bench.CONFIG.update(path=path, heads=2, grid=(6, 12, 16))
    inp, S = bench.make_layer_inputs(torch.device("cpu"))
    assert S == 6 * 12 * 16
    r = bench.CpuLayerSample(inp, S).run(seconds=1.0)
    assert r["value"] > 0 and r["kind"] == "port" and r["cores"] >= 1
    assert 0.0 < r["sample_pair_density"] <= 1.0
    if path == "uniform":
        assert abs(r["sample_pair_density"] - 0.25) < 0.05  # sparsity 0.75 on every q chunk
        assert "uniform 3D-chunk order" in r["sample"]
    else:
        assert "zone statistics" in r["sample"]
