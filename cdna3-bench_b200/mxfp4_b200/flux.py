"""The FLUX.1-dev double-stream block's linear sequence on the library's GEMMs.

BASELINE configs[1] names four linears of one FLUX.1-dev double-stream transformer block at
M = 4608 tokens: QKV (9216 x 3072), attention output (3072 x 3072), MLP up (12288 x 3072) and
MLP down (3072 x 12288).  :class:`FluxChain` runs them chained as the block uses them:

    qkv  = x @ W_qkv^T
    a    = qkv[:, :3072]               (stand-in for attention, which is out of scope here)
    h    = x + a @ W_out^T             (residual)
    u    = gelu_tanh(h @ W_up^T)
    out  = h + u @ W_down^T            (residual)

with bf16 activations between the steps (each GEMM writes bf16, accumulates fp32) and torch
element-wise ops for the residuals and the GELU.  Every op writes into buffers allocated once,
so one forward can be captured in a CUDA graph and replayed.  :func:`reference_rows` is the same
sequence in fp32 on the CPU for a subset of rows (the chain is row-wise, so any row's output
depends on that row's input only): the parity check of the chain.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from . import kernels as kk


class FluxChain:
    """x0 [M, d] bf16 and weights (QKV, attn-out, MLP-up, MLP-down) as MXFP4Weight."""

    def __init__(self, weights, x0: torch.Tensor):
        w_qkv, w_out, w_up, w_down = weights
        M, d = x0.shape
        if not (w_qkv.K == d and w_out.K == d and w_out.N == d and w_up.K == d and w_down.K == w_up.N
                and w_down.N == d and w_qkv.N >= d):
            raise ValueError("FluxChain: weight shapes do not form a block over x0")
        self.w = (w_qkv, w_out, w_up, w_down)
        self.x0 = x0
        dev = x0.device
        self.qkv = torch.empty((M, w_qkv.N), dtype=torch.bfloat16, device=dev)
        self.attn_in = torch.empty((M, d), dtype=torch.bfloat16, device=dev)
        self.attn_out = torch.empty((M, d), dtype=torch.bfloat16, device=dev)
        self.h = torch.empty((M, d), dtype=torch.bfloat16, device=dev)
        self.up = torch.empty((M, w_up.N), dtype=torch.bfloat16, device=dev)
        self.act = torch.empty((M, w_up.N), dtype=torch.bfloat16, device=dev)
        self.down = torch.empty((M, d), dtype=torch.bfloat16, device=dev)
        self.out = torch.empty((M, d), dtype=torch.bfloat16, device=dev)

    def forward(self, events=None) -> torch.Tensor:
        """One pass; `events` (optional) is a list of four (start, end) CUDA event pairs
        recorded around the four GEMMs."""

        def g(j, a, c):
            if events is not None:
                events[j][0].record()
            kk.gemm(a, self.w[j], C=c)
            if events is not None:
                events[j][1].record()
            return c

        d = self.x0.shape[1]
        g(0, self.x0, self.qkv)
        self.attn_in.copy_(self.qkv[:, :d])
        g(1, self.attn_in, self.attn_out)
        torch.add(self.x0, self.attn_out, out=self.h)
        g(2, self.h, self.up)
        self.act.copy_(F.gelu(self.up, approximate="tanh"))
        g(3, self.act, self.down)
        torch.add(self.h, self.down, out=self.out)
        return self.out


def _bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest bf16 (ties to even), returned as fp32."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def reference_rows(x0_rows: np.ndarray, dequantized, round_bf16: bool = True) -> np.ndarray:
    """The chain on the CPU in fp32 for some rows of x0 (fp32 values of the bf16 input).
    `dequantized`: the four weights as fp32 [K, N] arrays (A @ W layout, e.g. the oracle's
    dequantize_mxfp4 of the reference-layout bytes).  With `round_bf16` the intermediates are
    rounded to bf16 where the GPU chain stores bf16, so the remaining difference is the fp32
    accumulation order alone."""
    w_qkv, w_out, w_up, w_down = dequantized
    r = _bf16 if round_bf16 else (lambda v: v.astype(np.float32))
    x = x0_rows.astype(np.float32)
    d = x.shape[1]
    qkv = r(x @ w_qkv)
    a = qkv[:, :d]
    h = r(x + r(a @ w_out))
    u = r(h @ w_up)
    c = math.sqrt(2.0 / math.pi)
    act = r(0.5 * u * (1.0 + np.tanh(c * (u + 0.044715 * u * u * u))))
    return r(h + r(act @ w_down))
