"""GPU parity of the opt-in block-scaled path (MXFP8 activations x MXFP4 weights on the
tensor cores' block-scaled MMA) against its oracle: byte-exact activation quantisation and
weight re-layout, and the GEMM within max|err|/max|ref| <= 1e-2 of dequant(Q8(A)) @ dequant(W).

These tests run only with MXFP4_MX_GPU_TESTS=1: the path is built and its host logic is tested
on CPU, but it has not yet had its first run on a B200, which is done deliberately, alone, on
the smallest case before it joins the default GPU suite.
"""

import os

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import make_case, rel_err

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("MXFP4_MX_GPU_TESTS") != "1",
                       reason="block-scaled path: set MXFP4_MX_GPU_TESTS=1 to run its GPU tests"),
]


@pytest.fixture(scope="module")
def mx():
    import mxfp4_b200

    return mxfp4_b200


@pytest.fixture(autouse=True)
def _no_device_error(mx):
    mx.device_error(clear=True)
    yield
    torch.cuda.synchronize()
    assert mx.device_error(clear=True) == 0


@pytest.mark.parametrize("M,K", [(1, 128), (300, 160), (512, 3072)])
def test_act_quant_matches_oracle(mx, M, K):
    rng = np.random.default_rng(M + K)
    A = (rng.standard_normal((M, K)) * np.exp2(rng.integers(-12, 12, size=(M, 1)))).astype(np.float32)
    A[0, :32] = 0.0  # an all-zero group
    Ab = torch.from_numpy(A).to(torch.bfloat16)
    c, s = o.quantize_act_mx8(Ab.float().numpy())
    want_codes, want_blocks = o.mx_act_layout(c, s)
    codes, blocks = mx.quantize_act_mx8(Ab.cuda())
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(blocks.cpu().numpy(), want_blocks)


@pytest.mark.parametrize("N,K", [(128, 128), (200, 224), (3072, 3072)])
def test_weight_prepack_matches_oracle(mx, N, K):
    _, Bp, Bs = make_case(1, N, K, seed=N)
    w = mx.prepack_mx(Bp, Bs)
    np.testing.assert_array_equal(w.data.cpu().numpy(), o.mx_weight_layout(Bp, Bs))
    w_nk = mx.prepack_mx(np.ascontiguousarray(Bp.T), np.ascontiguousarray(Bs.T), layout="nk")
    assert torch.equal(w_nk.data, w.data)


@pytest.mark.parametrize("M,N,K", [(256, 128, 128), (300, 200, 224), (1024, 1024, 1024), (16, 384, 512)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_mx_matches_oracle(mx, M, N, K, out_dtype):
    A, Bp, Bs = make_case(M, N, K, seed=M * 7 + N)
    ref = o.ref_gemm_mx(A, Bp, Bs)
    w = mx.prepack_mx(Bp, Bs)
    C = mx.gemm_mx(torch.from_numpy(A).to(torch.bfloat16).cuda(), w, out_dtype=out_dtype)
    assert rel_err(C.float().cpu().numpy(), ref) <= 1e-2


def test_gemm_mx_flux_qkv_rows(mx):
    M, N, K = 4608, 9216, 3072
    A, Bp, Bs = make_case(M, N, K, seed=11)
    w = mx.prepack_mx(Bp, Bs)
    C = mx.gemm_mx(torch.from_numpy(A).to(torch.bfloat16).cuda(), w).float().cpu().numpy()
    rows = np.r_[0:64, 2300:2364, M - 64:M]
    ref = o.ref_gemm_mx(A[rows], Bp, Bs)
    assert rel_err(C[rows], ref) <= 1e-2
