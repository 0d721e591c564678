"""Parity at the full sizes of every benchmark configuration, against the CPU oracle.

Every GEMM shape the benchmark configurations name runs at its full size on the GPU:
  c0                 M = 128,  N = K = 3072;
  FLUX double-stream M = 4608, (N, K) in (9216, 3072), (3072, 3072), (12288, 3072), (3072, 12288);
  FLUX single-stream M = 4608, (N, K) in (21504, 3072), (3072, 15360);
  decode             M in (1, 4, 16), (N, K) in (10240, 8192), (8192, 8192), (57344, 8192), (8192, 28672).
The output of the library's default path (bf16 and fp32 C, weights prepacked once) and of the
one-call reference-layout entry (gemm_packed) is compared, on sampled rows (first, middle, last
and seeded random ones) and sampled output columns (whole first, middle and last 128-column
tiles plus seeded random columns), with the CPU oracle of the reference's ref_gemm
(oracle.ref_gemm: NumPy dequant + fp32 matmul) on the same bytes: max|err|/max|ref| <= 1e-2 and
the reference's own np.allclose(atol=1e-2, rtol=2e-2).  Weights and activations follow the
benchmark's generation (N(0, 0.02) weights, OCP-MXFP4-quantised along K on the GPU; the GPU
quantiser is byte-identical to the oracle's, tested in test_gpu_formats.py).
"""

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import rel_err

pytestmark = pytest.mark.gpu

TOL = 1e-2

FLUX = [(9216, 3072), (3072, 3072), (12288, 3072), (3072, 12288), (21504, 3072), (3072, 15360)]
DECODE = [(10240, 8192), (8192, 8192), (57344, 8192), (8192, 28672)]


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


def _weights(mx, N, K, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    W = torch.randn((K, N), generator=g, device="cuda") * 0.02
    Bp, Bs = mx.quantize_mxfp4(W, axis=0, rule="ocp")  # reference layout [K/2, N], [K/32, N]
    del W
    return Bp, Bs


def _sample(n, tile, seed, count):
    """Whole first, middle and last tiles plus `count` seeded random indices, sorted, unique."""
    rng = np.random.default_rng(seed)
    mid = (n // 2) // tile * tile
    idx = np.r_[0:min(tile, n), mid:min(mid + tile, n), max(0, n - tile):n, rng.integers(0, n, size=count)]
    return np.unique(idx)


def _check(out_gpu: torch.Tensor, rows, cols, ref):
    got = out_gpu[torch.as_tensor(rows, device="cuda")][:, torch.as_tensor(cols, device="cuda")].float().cpu().numpy()
    assert rel_err(got, ref) <= TOL
    assert np.allclose(got, ref, atol=1e-2, rtol=2e-2)


def _run_shape(mx, Ms, N, K, seed):
    Bp, Bs = _weights(mx, N, K, seed)
    cols = _sample(N, 128, seed + 1, 256)
    Bp_c, Bs_c = Bp[:, cols].cpu().numpy(), Bs[:, cols].cpu().numpy()  # the sampled columns' bytes
    w = mx.prepack_b200(Bp, Bs)
    g = torch.Generator(device="cuda").manual_seed(seed + 2)
    for M in Ms:
        A = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        rows = np.arange(M) if M <= 64 else _sample(M, 16, seed + M, 16)
        ref = o.ref_gemm(A[torch.as_tensor(rows, device="cuda")].float().cpu().numpy(), Bp_c, Bs_c)
        _check(mx.gemm(A, w, out_dtype=torch.bfloat16), rows, cols, ref)
        _check(mx.gemm(A, w, out_dtype=torch.float32), rows, cols, ref)
        _check(mx.gemm_packed(A, Bp, Bs, out_dtype=torch.float32), rows, cols, ref)
        del A
    torch.cuda.synchronize()


def test_c0_full_size(mx):
    _run_shape(mx, [128], 3072, 3072, seed=100)


@pytest.mark.parametrize("N,K", FLUX)
def test_flux_full_size(mx, N, K):
    _run_shape(mx, [4608], N, K, seed=N + K)


@pytest.mark.parametrize("N,K", DECODE)
def test_decode_full_size(mx, N, K):
    _run_shape(mx, [1, 4, 16], N, K, seed=N + 3 * K)
