"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (pure NumPy, no GPU):

    python tests/golden/make_golden.py --ref-python <reference>/python

It imports the reference's own ``mxfp4_cdna3.ref`` module (ref.py) and stores
its outputs on seeded inputs in ``tests/golden/ref_vectors.npz``.  The tests
only read the .npz, so neither the reference nor this script is needed where
the tests run.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np


def tie_heavy(rng, shape):
    """Values that land exactly on E2M1 midpoints after scaling (scale 2**0 blocks)."""
    mids = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 6.0, 0.0, 0.5, 3.0, 4.0], np.float32)
    x = rng.choice(mids, size=shape) * rng.choice(np.array([-1, 1], np.float32), size=shape)
    # force every 32-block along the last axis to have amax exactly 6 -> exponent 0
    x.reshape(-1, 32)[:, 0] = 6.0
    return x.astype(np.float32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-python", required=True)
    ap.add_argument("--out", default=str(Path(__file__).with_name("ref_vectors.npz")))
    args = ap.parse_args()
    sys.path.insert(0, args.ref_python)
    from mxfp4_cdna3 import ref as rr  # the reference's own module

    rng = np.random.default_rng(20240601)
    out = {}

    # 1. quantiser, along axis 0 ([K, N] weights, as validate.py uses it) and axis -1
    cases = {
        "normal": rng.standard_normal((128, 96), dtype=np.float32) * 0.1,
        "wide": (rng.standard_normal((64, 64), dtype=np.float32)
                 * np.exp2(rng.integers(-40, 40, size=(64, 64))).astype(np.float32)),
        "ties": tie_heavy(rng, (64, 64)),
        "tiny": rng.standard_normal((64, 32), dtype=np.float32) * np.float32(1e-39),
        "zeros": np.zeros((32, 32), np.float32),
        "w002": rng.standard_normal((256, 64), dtype=np.float32) * 0.02,
    }
    for name, x in cases.items():
        for ax in (0, -1):
            p, s = rr.quantize_mxfp4(x, axis=ax)
            tag = f"q_{name}_ax{ax % 2}"
            out[tag + "_x"] = x
            out[tag + "_p"] = p
            out[tag + "_s"] = s

    # 2. dequantiser on random bytes with every scale value 0..255 (axis 0 = [K/2, N])
    K, N = 32 * 8, 256
    p = rng.integers(0, 256, size=(K // 2, N), dtype=np.uint8)
    s = np.tile(np.arange(256, dtype=np.uint8), (K // 32, 1))[:, :N]
    s = np.ascontiguousarray(np.roll(s, 3, axis=1))
    with np.errstate(all="ignore"):
        d = rr.dequantize_mxfp4(p, s, axis=0)
    out["dq_p"], out["dq_s"], out["dq_out"] = p, s, d.astype(np.float32)

    # 3. ref_gemm on validate.py-style inputs (seed 42 style, 0.1 * N(0,1))
    M, N, K = 64, 128, 256
    A = (rng.standard_normal((M, K), dtype=np.float32) * 0.1).astype(np.float32)
    B = rng.standard_normal((K, N), dtype=np.float32) * 0.1
    Bp, Bs = rr.quantize_mxfp4(B, axis=0)
    out["gemm_A"], out["gemm_Bp"], out["gemm_Bs"] = A, Bp, Bs
    out["gemm_C"] = rr.ref_gemm(A, Bp, Bs).astype(np.float32)

    # 4. strategy-G prepack layout
    Bp2, Bs2 = rr.quantize_mxfp4(rng.standard_normal((128, 256), dtype=np.float32), axis=0)
    gp, gs = rr.prepack_b_mxfp4(Bp2, Bs2)
    out["g_Bp"], out["g_Bs"], out["g_prep"], out["g_sprep"] = Bp2, Bs2, gp, gs

    np.savez_compressed(args.out, **out)
    print(f"wrote {args.out}: {len(out)} arrays")


if __name__ == "__main__":
    main()
