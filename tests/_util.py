"""Shared helpers for the tests: golden vectors, seeded inputs, error metrics."""

import os

import numpy as np

import mxfp4_ref as oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_vectors.npz")


def golden():
    return np.load(GOLDEN)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to bf16 (RNE), returned as fp32."""
    return oracle.bf16_bits_to_f32(oracle.f32_to_bf16_bits(x))


def make_case(M, N, K, seed=0, w_std=0.02, rule="ocp", a_std=1.0):
    """Synthetic inputs in the benchmark's distribution: A ~ N(0, a_std) rounded to bf16,
    W ~ N(0, w_std) of [N, K] quantised along K, returned in the reference layout."""
    rng = np.random.default_rng(seed)
    A = bf16_round(rng.standard_normal((M, K), dtype=np.float32) * np.float32(a_std))
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(w_std)
    q = oracle.quantize_mxfp4_ocp if rule == "ocp" else oracle.quantize_mxfp4
    Bp, Bs = q(W, axis=0)
    return A, Bp, Bs


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max|err| / max|ref| (the parity bar: <= 1e-2)."""
    return float(np.max(np.abs(out.astype(np.float64) - ref)) / max(np.max(np.abs(ref)), 1e-30))
