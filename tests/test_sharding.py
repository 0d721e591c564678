"""Column-parallel (N-sharded) host logic: slice bounds, weight slicing and the all-gather
assembly, run as two gloo ranks on CPU.  The per-rank GEMM is the CPU oracle here (the
GPU kernel is covered by the gpu-marked tests); what is under test is that the slices tile
N exactly and that the gathered output equals the unsharded product."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import mxfp4_ref as o
from mxfp4_b200 import sharding


def test_column_slice_tiles_exactly():
    for N in (128, 384, 3072, 7168, 57344, 128 * 13):
        for world in (1, 2, 3, 4, 8):
            if N // 128 < world:
                with pytest.raises(ValueError):
                    sharding.column_slice(N, world, 0)
                continue
            bounds = [sharding.column_slice(N, world, r) for r in range(world)]
            assert bounds[0][0] == 0 and bounds[-1][1] == N
            for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
                assert a1 == b0
            sizes = [b - a for a, b in bounds]
            assert all(s % 128 == 0 and s > 0 for s in sizes)
            assert max(sizes) - min(sizes) <= 128
    with pytest.raises(ValueError):
        sharding.column_slice(200, 2, 0)
    with pytest.raises(ValueError):
        sharding.column_slice(256, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, N, K, M, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        A, Bp, Bs = _case(M, N, K)
        bp, bs = sharding.shard_reference_weights(torch.from_numpy(Bp), torch.from_numpy(Bs), world, rank)
        n0, n1 = sharding.column_slice(N, world, rank)
        assert bp.shape == (K // 2, n1 - n0) and bs.shape == (K // 32, n1 - n0)
        Y = torch.from_numpy(o.ref_gemm(A, bp.numpy(), bs.numpy()))
        full = sharding.all_gather_columns(Y, N)
        q.put((rank, full.numpy()))
    finally:
        dist.destroy_process_group()


def _case(M, N, K):
    rng = np.random.default_rng(7)
    A = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(0.02)
    Bp, Bs = o.quantize_mxfp4_ocp(W, axis=0)
    return A, Bp, Bs


@pytest.mark.parametrize("N", [512, 640])  # equal slices, and unequal (5 tiles over 2 ranks)
def test_gloo_two_ranks_gather_equals_unsharded(N):
    M, K, world = 8, 128, 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, N, K, M, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    A, Bp, Bs = _case(M, N, K)
    ref = o.ref_gemm(A, Bp, Bs)
    for r in range(world):
        np.testing.assert_allclose(results[r], ref, rtol=1e-6, atol=1e-6)
