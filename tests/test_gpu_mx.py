"""GPU parity of the block-scaled paths (E4M3-coded activations x MXFP4 weights on the tensor
cores' block-scaled MMA) against their oracle: byte-exact activation coding (both modes) and
weight re-layout, the GEMM within max|err|/max|ref| <= 1e-2 of (sum of the dequantised
activation pieces) @ dequant(W), and the split2 mode within the same bar of the exact product.

The path's first GPU run followed a staged order (coder and prepack alone, then one small GEMM
per kernel, then this whole file), with programmatic dependent launch off (MXFP4_NO_PDL=1) and
then on; every stage passed, so these tests are part of the default GPU suite.
"""

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import make_case, rel_err

pytestmark = pytest.mark.gpu


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


MODES = {"q8": o.MX_Q8, "split2": o.MX_SPLIT2}


@pytest.mark.parametrize("mode", ["q8", "split2"])
@pytest.mark.parametrize("M,K", [(1, 128), (16, 160), (300, 160), (512, 3072)])
def test_act_coding_matches_oracle(mx, M, K, mode):
    rng = np.random.default_rng(M + K)
    A = (rng.standard_normal((M, K)) * np.exp2(rng.integers(-12, 12, size=(M, 1)))).astype(np.float32)
    A[0, :32] = 0.0  # an all-zero group
    Ab = torch.from_numpy(A).to(torch.bfloat16)
    want_codes, want_blocks = o.mx_act_layout(Ab.float().numpy(), MODES[mode])
    codes, blocks = mx.quantize_act_mx8(Ab.cuda(), mode)
    np.testing.assert_array_equal(codes.cpu().numpy(), want_codes)
    np.testing.assert_array_equal(blocks.cpu().numpy(), want_blocks)


@pytest.mark.parametrize("N,K", [(128, 128), (200, 224), (3072, 3072)])
def test_weight_prepack_matches_oracle(mx, N, K):
    _, Bp, Bs = make_case(1, N, K, seed=N)
    w = mx.prepack_mx(Bp, Bs)
    np.testing.assert_array_equal(w.data.cpu().numpy(), o.mx_weight_layout(Bp, Bs))
    w_nk = mx.prepack_mx(np.ascontiguousarray(Bp.T), np.ascontiguousarray(Bs.T), layout="nk")
    assert torch.equal(w_nk.data, w.data)


@pytest.mark.parametrize("mode", ["q8", "split2"])
@pytest.mark.parametrize("M,N,K", [(256, 128, 128), (300, 200, 224), (1024, 1024, 1024), (1, 384, 512),
                                   (16, 10240, 1024), (7, 200, 224)])
@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_gemm_mx_matches_oracle(mx, M, N, K, mode, out_dtype):
    A, Bp, Bs = make_case(M, N, K, seed=M * 7 + N)
    ref = o.ref_gemm_mx(A, Bp, Bs, MODES[mode])
    w = mx.prepack_mx(Bp, Bs)
    C = mx.gemm_mx(torch.from_numpy(A).to(torch.bfloat16).cuda(), w, out_dtype=out_dtype, mode=mode)
    assert rel_err(C.float().cpu().numpy(), ref) <= 1e-2


@pytest.mark.parametrize("M", [1, 16, 4608])
def test_gemm_split2_within_exact_bar(mx, M):
    """split2 against the EXACT reference (bf16 activations, dequantised weights): the same
    max|err|/max|ref| <= 1e-2 bar as the exact path."""
    N, K = 3072, 3072
    A, Bp, Bs = make_case(M, N, K, seed=5)
    w = mx.prepack_mx(Bp, Bs)
    C = mx.gemm_mx(torch.from_numpy(A).to(torch.bfloat16).cuda(), w, mode="split2").float().cpu().numpy()
    rows = np.r_[0:min(M, 64), max(0, M - 64):M]
    exact = A[rows] @ o.dequantize_mxfp4(Bp, Bs, axis=0)
    assert rel_err(C[rows], exact) <= 1e-2


def test_gemm_mx_flux_qkv_rows(mx):
    M, N, K = 4608, 9216, 3072
    A, Bp, Bs = make_case(M, N, K, seed=11)
    w = mx.prepack_mx(Bp, Bs)
    C = mx.gemm_mx(torch.from_numpy(A).to(torch.bfloat16).cuda(), w).float().cpu().numpy()
    rows = np.r_[0:64, 2300:2364, M - 64:M]
    ref = o.ref_gemm_mx(A[rows], Bp, Bs)
    assert rel_err(C[rows], ref) <= 1e-2
