"""The package's validate and sweep harnesses (mirrors of the reference's validate.py and
bench.py) and the column-parallel layer, run on the GPU."""

import csv

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import make_case, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(256, 256, 128), (16, 384, 256), (1, 1024, 512)])
def test_validate_shape(shape):
    from mxfp4_b200 import validate

    assert validate.validate_shape(*shape)


def test_validate_cli_exit_code():
    from mxfp4_b200 import validate

    with pytest.raises(SystemExit) as e:
        validate.main(["--shapes", "128,256,128", "--log-level", "WARNING"])
    assert e.value.code == 0


def test_sweep_writes_samples(tmp_path):
    from mxfp4_b200 import bench

    out = tmp_path / "sweep.csv"
    rows = bench.run_sweep([(128, 384, 256), (4, 512, 256)], out, n_warmup=2, n_iter=3, rot=2)
    with open(out) as f:
        got = list(csv.DictReader(f))
    assert len(got) == len(rows) > 0
    labels = {r["strategy"] for r in got}
    assert {"A", "AUTO", "G", "b200:tc"} <= labels and "b200:gemv" in labels
    assert all(float(r["ns"]) > 0 and float(r["frac_roofline"]) > 0 for r in got)
    med = bench.summarize(rows)
    assert ("AUTO", 128, 384, 256) in med


def test_column_parallel_single_process_slices():
    """Each rank's slice, computed with the GPU kernel, equals the matching columns of the
    full product; concatenated in rank order they give the whole output."""
    from mxfp4_b200 import sharding

    M, N, K, world = 64, 640, 256, 2
    A, Bp, Bs = make_case(M, N, K, seed=5)
    At = torch.from_numpy(A).cuda().to(torch.bfloat16)
    ref = o.ref_gemm(A, Bp, Bs)
    parts = []
    for r in range(world):
        layer = sharding.ColumnParallelMXFP4(torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda(), N, world, r)
        Y = layer.forward(At, gather=False, out_dtype=torch.float32)
        n0, n1 = layer.n0, layer.n1
        assert rel_err(Y.cpu().numpy(), ref[:, n0:n1]) <= 1e-2
        parts.append(Y)
    full = sharding.assemble(parts, N).cpu().numpy()
    assert rel_err(full, ref) <= 1e-2


def test_quantize_bench_runs():
    from mxfp4_b200 import bench

    rows = bench.bench_quantize([(256, 384)], n_iter=2)
    assert rows[0]["quantize_gbs"] > 0 and rows[0]["prepack_gbs"] > 0
