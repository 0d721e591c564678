"""CPU reference product for the validation harness, in NumPy.

The reference package ships its own CPU checker next to its kernels (python/mxfp4_cdna3/ref.py:
``dequantize_mxfp4`` :50-72 and ``ref_gemm`` :75-78), and its validation harness compares every
GPU strategy with that CPU product (validate.py:29-34).  This module is the same checker for
this package: the exact fp32 value of every weight, then an fp32 BLAS matmul, all on the host.
It is independent of the GPU code it checks: nothing here calls the library.

Bytes: E2M1 nibble = sign<<3 | magnitude index (magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6), the
even k in the low nibble; one E8M0 byte per 32 k, value 2**(byte - 127) (byte 255 is +inf in
fp32, so 0 * inf gives NaN as in the reference).
"""

from __future__ import annotations

import numpy as np

_MAG = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
_NIB = np.concatenate([_MAG, -_MAG]).astype(np.float32)  # value of each 4-bit code
# value pair (low nibble, high nibble) of every byte
_BYTE_PAIR = np.stack([np.repeat(_NIB[None, :], 16, 0).reshape(-1),  # low nibble = b & 15
                       np.repeat(_NIB, 16)], axis=1).astype(np.float32)  # high nibble = b >> 4


def dequantize_ref_layout(B_packed: np.ndarray, B_scales: np.ndarray) -> np.ndarray:
    """Reference-layout weights (packed uint8 [K/2, N], scales uint8 [K/32, N]) -> fp32 [K, N]."""
    Bp = np.asarray(B_packed, dtype=np.uint8)
    Bs = np.asarray(B_scales, dtype=np.uint8)
    K2, N = Bp.shape
    if Bs.shape != (2 * K2 // 32, N):
        raise ValueError("B_scales must be [K/32, N] for B_packed [K/2, N]")
    pairs = _BYTE_PAIR[Bp]                                   # [K/2, N, 2]: rows 2j, 2j+1
    vals = pairs.transpose(0, 2, 1).reshape(2 * K2, N)       # [K, N]
    with np.errstate(over="ignore"):
        mult = np.ldexp(np.float32(1.0), Bs.astype(np.int32) - 127).astype(np.float32)  # [K/32, N]
    with np.errstate(invalid="ignore", over="ignore"):
        return (vals.reshape(-1, 32, N) * mult[:, None, :]).reshape(2 * K2, N)


def ref_gemm(A: np.ndarray, B_packed: np.ndarray, B_scales: np.ndarray) -> np.ndarray:
    """fp32 A[M, K] @ dequant(B)[K, N] on the CPU."""
    A32 = np.asarray(A, dtype=np.float32)
    return A32 @ dequantize_ref_layout(B_packed, B_scales)
