"""Repeated large-M calls give bitwise-identical results.

The large-M kernel without split-K is deterministic (each output element is one TMEM accumulator,
summed in a fixed order), so every repetition must match the first bit for bit.  This guards the
hand-off between the weight-stage ring and the two dequant warp groups (gemm_tc_kernel): a group
uses each stage only every second phase of its barrier, and a race there once made about one
call in 150 compute a whole tile from a stale weight chunk -- values slightly off, no error word.
The first result is also checked against the CPU oracle on sampled rows, so "identical" cannot
mean "identically wrong".
"""

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_repeated_calls_bitwise_identical(dtype):
    import mxfp4_b200 as mx

    M, N, K, reps = 4608, 9216, 3072, 400  # FLUX QKV
    g = torch.Generator(device="cuda").manual_seed(11)
    W = torch.randn((K, N), generator=g, device="cuda") * 0.02
    Bp, Bs = mx.quantize_mxfp4(W, axis=0, rule="ocp")
    del W
    w = mx.prepack_b200(Bp, Bs)
    A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    mx.device_error(clear=True)
    first = mx.gemm(A, w, out_dtype=dtype).clone()
    rows = np.unique(np.r_[0:8, 2300:2308, M - 8:M])
    cols = np.unique(np.r_[0:256, N - 256:N])
    ref = o.ref_gemm(A[torch.as_tensor(rows, device="cuda")].float().cpu().numpy(), Bp[:, cols].cpu().numpy(),
                     Bs[:, cols].cpu().numpy())
    got = first[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")].float().cpu().numpy()
    assert rel_err(got, ref) <= 1e-2
    C = torch.empty_like(first)
    bad = []
    for i in range(reps):
        C.fill_(float("nan"))
        mx.gemm(A, w, C=C)
        if not torch.equal(C, first):
            bad.append(i)
    torch.cuda.synchronize()
    assert mx.device_error(clear=True) == 0
    assert not bad, f"{len(bad)} of {reps} calls differ from the first (first: call {bad[0]})"
