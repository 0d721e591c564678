"""The chained FLUX.1 double-stream block (mxfp4_b200.flux.FluxChain, the sequence bench.py times
as flux_chain) against the same chain on the CPU from the oracle's dequantised weights.

Full size (M = 4608 tokens, hidden 3072, MLP 12288).  The chain is row-wise (every op acts on
each token row alone), so sampled rows of the final residual output are compared with the CPU
chain run on those rows only: fp32 matmuls on the oracle's dequantisation of the very bytes the
GPU multiplies.  The GPU keeps bf16 activations between the steps, so the bound is 2e-2 relative
(max|err| / max|ref|) against the all-fp32 chain, and 1e-2 against the CPU chain that rounds
its intermediates to bf16 at the same points.
"""

import numpy as np
import pytest
import torch

import mxfp4_ref as o
from _util import rel_err

pytestmark = pytest.mark.gpu

SHAPES = [(9216, 3072), (3072, 3072), (12288, 3072), (3072, 12288)]  # (N, K): qkv, out, up, down


@pytest.fixture(scope="module")
def mx():
    import mxfp4_b200

    return mxfp4_b200


def test_flux_chain_matches_cpu_chain(mx):
    from mxfp4_b200.flux import FluxChain, reference_rows

    M = 4608
    g = torch.Generator(device="cuda").manual_seed(7)
    weights, deq = [], []
    for N, K in SHAPES:
        W = torch.randn((K, N), generator=g, device="cuda") * 0.02
        Bp, Bs = mx.quantize_mxfp4(W, axis=0, rule="ocp")
        weights.append(mx.prepack_b200(Bp, Bs))
        deq.append(o.dequantize_mxfp4(Bp.cpu().numpy(), Bs.cpu().numpy(), axis=0))  # [K, N] fp32
        del W
    x0 = torch.randn((M, 3072), generator=g, device="cuda").to(torch.bfloat16)
    chain = FluxChain(weights, x0)
    out = chain.forward()
    torch.cuda.synchronize()
    assert mx.device_error() == 0
    rows = np.unique(np.r_[0:16, 2296:2312, M - 16:M, np.random.default_rng(1).integers(0, M, 16)])
    idx = torch.as_tensor(rows, device="cuda")
    got = out[idx].float().cpu().numpy()
    x_rows = x0[idx].float().cpu().numpy()
    assert rel_err(got, reference_rows(x_rows, deq, round_bf16=False)) <= 2e-2
    assert rel_err(got, reference_rows(x_rows, deq, round_bf16=True)) <= 1e-2
    # replaying the same forward from a CUDA graph (as bench.py does) gives the same output
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        chain.forward()
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(chain.out, first)
