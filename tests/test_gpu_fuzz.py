"""Seeded random shapes through every entry point family (parity bar max|err|/max|ref| <= 1e-2):
M from 1 to 600 (both kernel families and split-K), N any multiple of 8, K any multiple of 32."""

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import make_case, rel_err

pytestmark = pytest.mark.gpu

_rng = np.random.default_rng(2024)
SHAPES = [(int(_rng.choice([1, 2, 3, 5, 8, 13, 16, 17, 31, 64, 100, 255, 256, 257, 600])),
           int(_rng.integers(1, 257)) * 8, int(_rng.integers(1, 129)) * 32) for _ in range(24)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_random_shape(M, N, K):
    import mxfp4_b200 as mx

    A, Bp, Bs = make_case(M, N, K, seed=M * 131 + N * 7 + K)
    ref = o.ref_gemm(A, Bp, Bs)
    At = torch.from_numpy(A).to(torch.bfloat16).cuda()
    w = mx.prepack_b200(Bp, Bs)
    out = mx.gemm(At, w, out_dtype=torch.float32).cpu().numpy()  # prepacked, cost-model path
    assert rel_err(out, ref) <= 1e-2
    Bpt, Bst = torch.from_numpy(Bp).cuda(), torch.from_numpy(Bs).cuda()
    out2 = mx.gemm_auto(At, Bpt, Bst).cpu().numpy()  # reference layout, one call
    assert rel_err(out2, ref) <= 1e-2
    out3 = mx.gemm(At, w, out_dtype=torch.bfloat16).float().cpu().numpy()
    assert rel_err(out3, ref) <= 1e-2
    torch.cuda.synchronize()
    assert mx.device_error() == 0
