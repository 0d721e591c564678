"""The allocation-free GEMM entry point, mxfp4_gemm_noalloc.

It exists for callers that cannot allocate device memory themselves (their device memory is
owned by a custom allocator or pool, or allocating would synchronise a pipeline) and so
cannot hand mxfp4_gemm a workspace for re-laying the weights.  These tests call it through
the C ABI and compare it with mxfp4_gemm given a workspace and with the CPU oracle of the
reference's ref_gemm, twice in a row, since every call reuses the library's one fixed buffer.  This file is collected last on purpose.
"""

import ctypes

import numpy as np
import pytest
import torch

import mxfp4_ref as oracle
from _util import make_case, rel_err

TOL = 1e-2  # max|err| / max|ref|, as in the other GEMM tests


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_rejects_weights_beyond_its_buffer():
    from mxfp4_b200 import _lib

    lib = _lib.lib()
    # 8192 x 8192 MXFP4 weights re-laid need ~34 MiB > the 32 MiB buffer: refused up front
    rc = lib.mxfp4_gemm_noalloc(None, None, None, None, 1, 16, 8192, 8192, _lib.LAYOUT_REF, 0, None)
    assert rc == 1006
    assert "32 MiB" in _lib.error_string(rc)
    # prepacked weights need no buffer at all: that layout belongs to mxfp4_gemm
    assert lib.mxfp4_gemm_noalloc(None, None, None, None, 1, 16, 64, 64, _lib.LAYOUT_PREPACKED, 0, None) == 1000


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,layout", [(300, 1152, 640, "ref"), (8, 1024, 2048, "ref"), (256, 384, 512, "nk")])
def test_noalloc_matches_workspace_entry_point_twice(M, N, K, layout):
    import mxfp4_b200 as mx
    from mxfp4_b200 import _lib

    lib = _lib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):  # the second call sees the first call's leftovers in the buffer
        A, Bp, Bs = make_case(M, N, K, seed=17 * call + M + N)
        At = torch.from_numpy(A).to(torch.bfloat16).cuda()
        ref = oracle.ref_gemm(A, Bp, Bs)
        if layout == "nk":
            Bp, Bs = np.ascontiguousarray(Bp.T), np.ascontiguousarray(Bs.T)
        Bpt, Bst = torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda()
        want = mx.gemm_packed(At, Bpt, Bst, out_dtype=torch.float32, layout=layout)
        got = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
        rc = lib.mxfp4_gemm_noalloc(_p(At), _p(Bpt), _p(Bst), _p(got), _lib.DTYPE_F32, M, N, K,
                                    {"ref": _lib.LAYOUT_REF, "nk": _lib.LAYOUT_NK}[layout], _lib.PATH_AUTO, stream)
        assert rc == 0, _lib.error_string(rc)
        torch.cuda.synchronize()
        assert mx.device_error() == 0
        w, g = want.cpu().numpy(), got.cpu().numpy()
        assert not np.isnan(g).any()
        assert rel_err(g, w) <= TOL
        assert rel_err(g, ref) <= TOL  # and against the CPU oracle of the reference's ref_gemm
