"""The fused column-parallel GEMM + all-gather (mxfp4_gemm_allgather): every destination
receives this GPU's columns at the right offset, for both kernel families; on two GPUs the
gathered output equals the unsharded product."""

import os
import socket

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import make_case, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,path", [(256, "tc"), (300, "tc_smem"), (4, "gemv"), (16, "gemv")])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_multi_destination_single_gpu(M, path, dtype):
    """Three local buffers stand in for three GPUs' outputs: each gets the slice at n_off."""
    import mxfp4_b200 as mx
    from mxfp4_b200 import kernels as kk

    N, K, ldc, n_off = 384, 512, 1024, 512
    A, Bp, Bs = make_case(M, N, K, seed=3 + M)
    ref = o.ref_gemm(A, Bp, Bs)
    w = mx.prepack_b200(Bp, Bs)
    At = torch.from_numpy(A).cuda().to(torch.bfloat16)
    bufs = [torch.full((M, ldc), 7.0, dtype=dtype, device="cuda") for _ in range(3)]
    kk.gemm_allgather(At, w, [b.data_ptr() for b in bufs], n_off, ldc, out_dtype=dtype, path=path)
    torch.cuda.synchronize()
    assert mx.device_error() == 0
    for b in bufs:
        h = b.float().cpu().numpy()
        assert rel_err(h[:, n_off:n_off + N], ref) <= 1e-2
        assert (h[:, :n_off] == 7.0).all() and (h[:, n_off + N:] == 7.0).all()  # nothing outside the slice


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_single_destination_split_k_at_offset(dtype):
    """One destination at a non-zero column offset on a shape with few tiles (3 tiles, K = 2048):
    the large-M kernel splits K and the reduction writes the slice at n_off (the copy-engine
    multi-GPU form runs every rank's GEMM this way)."""
    import mxfp4_b200 as mx
    from mxfp4_b200 import kernels as kk

    M, N, K, ldc, n_off = 256, 384, 2048, 1024, 512
    A, Bp, Bs = make_case(M, N, K, seed=5)
    ref = o.ref_gemm(A, Bp, Bs)
    w = mx.prepack_b200(Bp, Bs)
    At = torch.from_numpy(A).cuda().to(torch.bfloat16)
    buf = torch.full((M, ldc), 7.0, dtype=dtype, device="cuda")
    kk.gemm_allgather(At, w, [buf.data_ptr()], n_off, ldc, out_dtype=dtype, path="tc")
    torch.cuda.synchronize()
    assert mx.device_error() == 0
    h = buf.float().cpu().numpy()
    assert rel_err(h[:, n_off:n_off + N], ref) <= 1e-2
    assert (h[:, :n_off] == 7.0).all() and (h[:, n_off + N:] == 7.0).all()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q, how):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from mxfp4_b200 import sharding

        res = {}
        for M in (512, 8):
            N, K = 1024, 768
            A, Bp, Bs = make_case(M, N, K, seed=21 + M)
            layer = sharding.ColumnParallelMXFP4(torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda(), N, world, rank)
            out = sharding.PeerOutput(M, N, torch.float32)
            At = torch.from_numpy(A).cuda().to(torch.bfloat16)
            for _ in range(2):  # twice: the buffer is reused
                Y = getattr(sharding, how)(layer, At, out)
            torch.cuda.synchronize()
            res[M] = rel_err(Y.cpu().numpy(), o.ref_gemm(A, Bp, Bs))
            dist.barrier()
            out.close()
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("how", ["forward_fused", "forward_copy_engine"])
def test_two_gpu_fused_allgather_equals_unsharded(how):
    """Both multi-GPU forms -- the all-gather fused into the epilogue, and the copy-engine push
    after a local GEMM -- give every rank the unsharded product."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q, how)) for r in range(2)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        for M, err in got[r].items():
            assert err <= 1e-2, (r, M, err)
