"""CPU tests of the C ABI: the library loads, exports every declared symbol, and the
non-compute entry points behave (no GPU needed)."""

import ctypes
import os
import re

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mxfp4_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(mxfp4_[a-z_0-9]+)\s*\(", text)))


@pytest.fixture(scope="module")
def L():
    from mxfp4_b200 import _lib

    return _lib


def test_exports_every_declared_symbol(L):
    lib = L.lib()
    syms = declared_symbols()
    assert len(syms) >= 13
    assert sorted(L.EXPORTED) == syms
    for s in syms:
        assert hasattr(lib, s), s


def test_abi_version_and_queries(L):
    lib = L.lib()
    assert lib.mxfp4_abi_version() == 1
    # 3072 x 3072: 24 x 48 chunks of 4352 bytes = packed + scales exactly
    assert lib.mxfp4_prepacked_bytes(3072, 3072) == 3072 * 3072 // 2 + 3072 * 3072 // 32
    assert lib.mxfp4_prepacked_bytes(200, 96) == 2 * 2 * 4352
    # prepacked weights need no workspace for large M (no GPU here, so no split-K plan); decode
    # shapes (M <= 16) get optional room for the stream-K decode kernel: the activations as f16
    # (128*M bytes per 64-k chunk), 256 bytes of row shifts and fp32 sums [M][N rounded to 128],
    # each part 256-byte aligned -- or at least the other decode kernels' prestaged activations
    # (one 2 KiB block per chunk plus 256 bytes)
    def al(x):
        return -(-x // 256) * 256

    def sk(M, N, K):
        nb, kb = -(-N // 128), -(-K // 64)
        return al(kb * 128 * M) + 256 + al(M * nb * 128 * 4)

    assert lib.mxfp4_gemm_workspace_bytes(32, 3072, 3072, L.LAYOUT_PREPACKED) == 0
    assert lib.mxfp4_gemm_workspace_bytes(8, 3072, 3072, L.LAYOUT_PREPACKED) == max(sk(8, 3072, 3072), 48 * 2048 + 256)
    assert lib.mxfp4_gemm_workspace_bytes(1, 3072, 3072, L.LAYOUT_PREPACKED) == max(sk(1, 3072, 3072), 48 * 2048 + 256)
    assert lib.mxfp4_gemm_workspace_bytes(16, 57344, 8192, L.LAYOUT_PREPACKED) == sk(16, 57344, 8192)
    assert lib.mxfp4_gemm_workspace_bytes(32, 3072, 3072, L.LAYOUT_REF) == lib.mxfp4_prepacked_bytes(3072, 3072)
    assert lib.mxfp4_select_path(1, 8192, 8192) == L.PATH_GEMV
    assert lib.mxfp4_select_path(16, 8192, 8192) == L.PATH_GEMV
    assert lib.mxfp4_select_path(4608, 9216, 3072) == L.PATH_TC
    assert lib.mxfp4_shape_supported(L.PATH_TC, 4608, 9216, 3072) == 1
    assert lib.mxfp4_shape_supported(L.PATH_GEMV, 17, 9216, 3072) == 0
    assert lib.mxfp4_shape_supported(L.PATH_TC, 128, 3072, 100) == 0  # K % 32
    assert lib.mxfp4_shape_supported(L.PATH_TC, 128, 3071, 128) == 0  # N % 8


def test_invalid_arguments_rejected_before_any_launch(L):
    lib = L.lib()
    P = ctypes.c_void_p
    # null pointers / bad enums come back as MXFP4_ERR_INVALID_ARGUMENT without touching CUDA
    assert lib.mxfp4_gemm(None, None, None, None, 0, 8, 8, 32, 0, 0, None, 0, None) == 1000
    assert lib.mxfp4_gemm(P(16), P(16), P(16), P(16), 7, 8, 8, 32, 0, 0, None, 0, None) == 1000
    assert lib.mxfp4_gemm(P(16), P(16), P(16), P(16), 0, 8, 8, 32, 9, 0, None, 0, None) == 1000
    assert lib.mxfp4_gemm(P(16), P(16), P(16), P(16), 0, 8, 8, 33, 0, 0, None, 0, None) == 1001
    assert lib.mxfp4_gemm(P(17), P(16), P(16), P(16), 0, 8, 8, 32, 3, 0, None, 0, None) == 1002
    assert lib.mxfp4_quantize(None, 32, 32, 0, 0, None, None, None) == 1000
    assert lib.mxfp4_quantize(P(16), 33, 32, 0, 0, P(16), P(16), None) == 1001
    assert lib.mxfp4_prepack(P(16), P(16), 100, 64, 2, P(16), None) == 1001  # G needs N % 128
    assert "workspace" in L.error_string(1003)


def test_python_cost_model_agrees_with_library_path_choice(L):
    """cost_model.pick_path (Python, the reference's cost_model.py counterpart) and the
    library's mxfp4_select_path pick the same kernel family on a grid of shapes."""
    from mxfp4_b200 import cost_model as cm

    names = {v: k for k, v in L.PATH_NAMES.items()}
    for M in (1, 2, 4, 8, 16, 17, 32, 64, 128, 256, 4608, 8192):
        for N, K in ((3072, 3072), (8192, 8192), (57344, 8192), (1024, 28672), (9216, 3072)):
            assert cm.pick_path(cm.Shape(M, N, K)) == names[L.lib().mxfp4_select_path(M, N, K)], (M, N, K)


@pytest.mark.parametrize("M,N,K", [(1, 10240, 8192), (16, 200, 224), (17, 3072, 3072), (4608, 9216, 3072),
                                   (300, 136, 96)])
def test_block_scaled_sizes_match_layouts(L, M, N, K):
    """Host arithmetic of the block-scaled path against the layouts the oracle restates."""
    import mxfp4_ref as o
    from mxfp4_b200 import kernels as kk

    lib = L.lib()
    Np, Kp = -(-N // 128) * 128, -(-K // 128) * 128
    assert lib.mxfp4_mx_weight_bytes(N, K) == Np * Kp // 2 + Np * Kp // 32
    for mode, name in ((o.MX_Q8, "q8"), (o.MX_SPLIT2, "split2")):
        G, rows = o.mx_act_rows(M, mode)
        assert kk.mx_code_rows(M, name) == rows
        rows_sf = -(-rows // 128) * 128
        codes = -(-(rows * Kp) // 256) * 256
        sf = rows_sf * Kp // 32
        acc = M * N * 4 if M <= 16 else 0
        assert lib.mxfp4_mx_workspace_bytes(M, N, K, mode) == codes + (-(-sf // 256) * 256) + acc
    assert lib.mxfp4_mx_workspace_bytes(M, N, K, 2) == 0  # unknown mode


def test_block_scaled_rejects_bad_arguments(L):
    lib = L.lib()
    p = ctypes.c_void_p(16)  # never dereferenced: argument checks fail first
    assert lib.mxfp4_gemm_mx(p, p, p, L.DTYPE_BF16, 4, 128, 100, L.MX_Q8, p, 1 << 20, None) == 1001  # K % 32
    assert lib.mxfp4_gemm_mx(p, p, p, L.DTYPE_BF16, 4, 100, 128, L.MX_Q8, p, 1 << 20, None) == 1001  # N % 8
    assert lib.mxfp4_gemm_mx(p, p, p, L.DTYPE_BF16, 4, 128, 128, 7, p, 1 << 20, None) == 1000  # mode
    assert lib.mxfp4_gemm_mx(p, p, p, L.DTYPE_BF16, 4, 128, 128, L.MX_Q8, p, 16, None) == 1003  # workspace
    assert lib.mxfp4_prepack_mx(p, p, 128, 128, L.LAYOUT_G, p, None) == 1000  # layout
    assert lib.mxfp4_quantize_act_mx8(p, 4, 100, L.MX_Q8, p, None) == 1001
