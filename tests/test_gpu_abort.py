"""The kernels' bounded waits and their abort path, exercised without any fault.

Every wait inside the kernels gives up after a limit, records an error code that the host reads
with mxfp4_device_error(), lets the copies in flight land, frees its tensor memory and returns.
Here a test hook (mxfp4_test_hooks) lowers the limit to 1 ms and makes the weight producer of
the large-M (tcgen05) and decode kernels issue nothing, so that their consumers' waits run out:
the launch must return, leave a wait error code, and the next ordinary launch on the same
context must run clean and match the CPU oracle (it could not even start if an aborted CTA had
kept its tensor memory).  Nothing faults, traps or hangs: the producer simply stays idle.
"""

import ctypes

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import make_case, rel_err

pytestmark = pytest.mark.gpu

WAIT_CODES = {0x101, 0x102, 0x103, 0x104, 0x105, 0x106}


@pytest.fixture(scope="module")
def mx():
    import mxfp4_b200

    return mxfp4_b200


@pytest.fixture
def hooks(mx):
    from mxfp4_b200 import _lib

    lib = _lib.lib()
    torch.cuda.synchronize()
    mx.device_error(clear=True)

    def set_(withhold, limit_ns=0):
        _lib.check(lib.mxfp4_test_hooks(int(withhold), ctypes.c_ulonglong(limit_ns)), "mxfp4_test_hooks")

    yield set_
    torch.cuda.synchronize()
    set_(0, 0)
    mx.device_error(clear=True)


def _abort_then_clean(mx, hooks, M, N, K, path, out_dtype):
    A, Bp, Bs = make_case(M, N, K, seed=M + N)
    At = torch.from_numpy(A).to(torch.bfloat16).cuda()
    w = mx.prepack_b200(torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda())
    hooks(1, 1_000_000)  # producers idle, waits give up after 1 ms
    mx.gemm(At, w, out_dtype=out_dtype, path=path)
    torch.cuda.synchronize()  # the launch returned
    code = mx.device_error(clear=True)
    assert code in WAIT_CODES, hex(code)
    hooks(0, 0)
    C = mx.gemm(At, w, out_dtype=out_dtype, path=path)
    torch.cuda.synchronize()
    assert mx.device_error(clear=True) == 0
    assert rel_err(C.float().cpu().numpy(), o.ref_gemm(A, Bp, Bs)) <= 1e-2


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_tc_kernel_abort_path(mx, hooks, out_dtype):
    _abort_then_clean(mx, hooks, 512, 640, 512, "tc", out_dtype)


@pytest.mark.parametrize("M", [1, 4, 16])
def test_gemv_kernel_abort_path(mx, hooks, M):
    _abort_then_clean(mx, hooks, M, 1024, 2048, "gemv", torch.bfloat16)


def test_allgather_epilogue_abort_path(mx, hooks):
    """The multi-destination bf16 epilogue (paired output slabs behind a named barrier): both
    warps of every pair must leave together when their wait gives up."""
    from mxfp4_b200 import kernels as kk

    M, N, K, ldc = 512, 512, 512, 1536
    A, Bp, Bs = make_case(M, N, K, seed=9)
    At = torch.from_numpy(A).to(torch.bfloat16).cuda()
    w = mx.prepack_b200(torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda())
    bufs = [torch.zeros((M, ldc), dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    hooks(1, 1_000_000)
    kk.gemm_allgather(At, w, [b.data_ptr() for b in bufs], 512, ldc, path="tc")
    torch.cuda.synchronize()
    assert mx.device_error(clear=True) in WAIT_CODES
    hooks(0, 0)
    kk.gemm_allgather(At, w, [b.data_ptr() for b in bufs], 512, ldc, path="tc")
    torch.cuda.synchronize()
    assert mx.device_error(clear=True) == 0
    ref = o.ref_gemm(A, Bp, Bs)
    for b in bufs:
        got = b[:, 512:1024].float().cpu().numpy()
        assert rel_err(got, ref) <= 1e-2
        assert not np.any(b[:, :512].float().cpu().numpy())  # nothing outside the slice
