"""The drop-in operator surface (names, argument meaning, error behaviour)."""

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


def test_reference_entry_points(mx):
    M, N, K = 256, 256, 128
    rng = np.random.default_rng(42)  # validate.py's generation
    A32 = rng.standard_normal((M, K), dtype=np.float32) * 0.1
    A = torch.from_numpy(A32).to(torch.bfloat16).cuda()
    B = rng.standard_normal((K, N), dtype=np.float32) * 0.1
    Bp_np, Bs_np = o.quantize_mxfp4(B, axis=0)
    Bp, Bs = torch.from_numpy(Bp_np).cuda(), torch.from_numpy(Bs_np).cuda()
    ref = o.ref_gemm(A.cpu().float().numpy(), Bp_np, Bs_np)
    for name in ("gemm_a", "gemm_b", "gemm_c", "gemm_d", "gemm_e", "gemm_f", "gemm_h", "gemm_i",
                 "gemm_j", "gemm_k", "gemm_m", "gemm_auto"):
        C = getattr(mx, name)(A, Bp, Bs)
        assert C.dtype == torch.float32 and tuple(C.shape) == (M, N), name
        assert np.allclose(C.cpu().numpy(), ref, atol=1e-2, rtol=2e-2), name
    gp, gs = mx.prepack_b_mxfp4(Bp_np, Bs_np)
    np.testing.assert_array_equal(gp, o.prepack_b_mxfp4(Bp_np, Bs_np)[0])
    C = mx.gemm_g(A, torch.from_numpy(gp).cuda(), torch.from_numpy(gs).cuda())
    assert np.allclose(C.cpu().numpy(), ref, atol=1e-2, rtol=2e-2)
    Cpre = torch.zeros((M, N), dtype=torch.float32, device="cuda")
    out = mx.gemm_j(A, Bp, Bs, Cpre)
    assert out.data_ptr() == Cpre.data_ptr()
    assert np.allclose(Cpre.cpu().numpy(), ref, atol=1e-2, rtol=2e-2)


def test_error_behaviour(mx):
    A, Bp, Bs = make_case(64, 128, 64)
    At = torch.from_numpy(A).to(torch.bfloat16).cuda()
    Bpt, Bst = torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda()
    with pytest.raises(RuntimeError, match="bfloat16"):
        mx.gemm_auto(At.float(), Bpt, Bst)
    with pytest.raises(RuntimeError, match="B_packed shape"):
        mx.gemm_auto(At, Bpt[:-1], Bst)
    with pytest.raises(RuntimeError, match="GPU"):
        mx.gemm_auto(At.cpu(), Bpt, Bst)
    with pytest.raises(RuntimeError, match="C must be float32"):
        mx.gemm_auto(At, Bpt, Bst, torch.empty((64, 128), dtype=torch.bfloat16, device="cuda"))
    with pytest.raises(RuntimeError, match="not supported"):
        mx.gemm(At, mx.prepack_b200(Bpt, Bst), path="gemv")  # M = 64 > 16


def test_ref_gemm_and_numpy_roundtrip(mx):
    A, Bp, Bs = make_case(32, 64, 64, rule="ref")
    C = mx.ref_gemm(A, Bp, Bs)
    assert isinstance(C, np.ndarray)
    assert rel_err(C, o.ref_gemm(A, Bp, Bs)) < 1e-5
    p, s = mx.quantize_mxfp4(np.array([[4.0, -4.0] * 16], dtype=np.float32), axis=-1)
    assert s[0, 0] == 127 and (p[0] == 0xE6).all()


def test_device_info_and_predicates(mx):
    d = mx.device_info(0)
    for key in ("name", "gcn_arch_name", "multi_processor_count", "total_global_mem",
                "shared_mem_per_block", "warp_size"):
        assert key in d
    assert d["gcn_arch_name"].startswith("sm_10")
    assert mx.shape_supported_c(4608, 9216, 3072)
    assert mx.select_path(4, 8192, 8192) == "gemv"
    assert mx.select_path(4608, 9216, 3072) == "tc"


def test_gemm_a_writes_fp32_accumulated_product(mx):
    """The unfused two-pass baseline writes the fp32-accumulated product like the reference's
    strategy A: far tighter than the 2**-9 relative step a bf16-rounded result would show."""
    M, N, K = 96, 640, 1024
    A, Bp, Bs = make_case(M, N, K, seed=3)
    ref = o.ref_gemm(A, Bp, Bs)
    C = mx.gemm_a(torch.from_numpy(A).to(torch.bfloat16).cuda(), torch.from_numpy(Bp).cuda(),
                  torch.from_numpy(Bs).cuda())
    assert C.dtype == torch.float32
    got = C.cpu().numpy()
    assert rel_err(got, ref) < 1e-5
    # a bf16-rounded output would miss the oracle by up to half a bf16 ulp of each element
    assert np.max(np.abs(got - ref) / np.maximum(np.abs(ref), 0.05)) < 2.0 ** -12
