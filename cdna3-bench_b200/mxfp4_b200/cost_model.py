"""Analytical B200 cost model for the MXFP4 x BF16 GEMM.

Replaces the reference's CDNA3 model (python/mxfp4_cdna3/cost_model.py:117-146 ``predict``,
``:153-167`` ``fit_efficiency``) with the two rooflines that bound this op on B200 and the
per-path efficiencies that pick a path:

    t_roof = max(2*M*N*K / P_bf16,  (N*K/2 + N*K/32 + M*K*2) / BW_hbm)

(the byte term is weights + scales + activations; the output M*N*2 is reported apart).
Peaks come from the driver's MEASURED_PEAKS.json when it exists.
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass

# Fallback peaks (an earlier measurement on this pool) when MEASURED_PEAKS.json is absent.
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0


@dataclass(frozen=True)
class Peaks:
    hbm_gbs: float
    bf16_tflops: float
    bf16_tflops_sustained: float
    source: str  # "measured" or "fallback"


def load_peaks(path: str | None = None) -> Peaks:
    here = os.path.dirname(os.path.abspath(__file__))
    cands = [path] if path else []
    cands.append(os.path.join(os.path.dirname(os.path.dirname(here)), "MEASURED_PEAKS.json"))
    for c in cands:
        if c and os.path.exists(c):
            with open(c) as f:
                d = json.load(f)
            return Peaks(float(d["hbm_gbs"]), float(d["bf16_tflops"]),
                         float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured")
    return Peaks(FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback")


@dataclass(frozen=True)
class Shape:
    M: int
    N: int
    K: int

    @property
    def flops(self) -> float:
        return 2.0 * self.M * self.N * self.K

    @property
    def weight_bytes(self) -> int:
        return self.N * self.K // 2 + self.N * self.K // 32

    @property
    def act_bytes(self) -> int:
        return self.M * self.K * 2

    @property
    def in_bytes(self) -> int:
        return self.weight_bytes + self.act_bytes

    @property
    def out_bytes_bf16(self) -> int:
        return self.M * self.N * 2


@dataclass(frozen=True)
class Roofline:
    t_compute_us: float
    t_hbm_us: float
    bound: str  # "tensor" or "hbm"

    @property
    def t_us(self) -> float:
        return max(self.t_compute_us, self.t_hbm_us)


def roofline(s: Shape, peaks: Peaks, sustained: bool = False) -> Roofline:
    p = peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops
    tc = s.flops / (p * 1e12) * 1e6
    th = s.in_bytes / (peaks.hbm_gbs * 1e9) * 1e6
    return Roofline(tc, th, "tensor" if tc >= th else "hbm")


# Efficiency of each path relative to its binding roofline, measured on B200 (refit with
# fit_efficiency from bench rows): the tcgen05 kernel runs the FLUX GEMMs at ~0.80 of the bf16
# peak; the decode kernel streams the decode shapes at ~0.35-0.65 of the HBM copy rate.
PATH_EFF = {"tc": 0.80, "gemv": 0.45}
TC_TILE_ACT = 256
TC_TILE_W = 128


def predict_us(path: str, s: Shape, peaks: Peaks, num_sms: int = 148) -> float:
    """Predicted kernel time of one path on one shape (~3 us launch overhead included)."""
    launch = 3.0
    if path == "gemv":
        if s.M > 16:
            return float("inf")
        return launch + s.in_bytes / (peaks.hbm_gbs * 1e9 * PATH_EFF["gemv"]) * 1e6
    m_tiles = -(-s.M // TC_TILE_ACT)
    n_tiles = -(-s.N // TC_TILE_W)
    waves = -(-(m_tiles * n_tiles) // num_sms)
    per_tile_flops = 2.0 * TC_TILE_ACT * TC_TILE_W * s.K
    per_sm_tflops = peaks.bf16_tflops * PATH_EFF["tc"] / num_sms
    t_c = waves * per_tile_flops / (per_sm_tflops * 1e12) * 1e6
    t_h = (s.weight_bytes + s.act_bytes) / (peaks.hbm_gbs * 1e9) * 1e6
    return launch + max(t_c, t_h)


def pick_path(s: Shape, peaks: Peaks | None = None, num_sms: int = 148) -> str:
    peaks = peaks or load_peaks()
    return min(("tc", "gemv"), key=lambda p: predict_us(p, s, peaks, num_sms))


def fit_efficiency(rows) -> dict:
    """rows: iterable of (path, M, N, K, measured_us) -> median achieved/roofline per path."""
    peaks = load_peaks()
    acc: dict = {}
    for path, M, N, K, us in rows:
        acc.setdefault(path, []).append(roofline(Shape(M, N, K), peaks).t_us / us)
    return {p: sorted(v)[len(v) // 2] for p, v in acc.items()}
