"""Validation harness: every entry point against an fp32 reference product, per shape.

    python -m mxfp4_b200.validate [--shapes M,N,K ...] [--log-level INFO]

Mirrors python/mxfp4_cdna3/validate.py:22-92 (validate_shape) and :95-110 (main): the same
seeded inputs (seed 42, A and W ~ 0.1*N(0,1), W quantised along K with the reference
rounding), the same acceptance rule np.allclose(atol=1e-2, rtol=2e-2) against fp32
A @ dequant(B), and the same list of strategy labels -- each label resolves to the B200 kernel
its entry point dispatches to.  On top of the reference's checks it runs each kernel family
explicitly (tcgen05 large-M "tc", "tc_smem", decode "gemv"), the bf16-output entry point, and
the bit-exact check of the dequantised tile the tensor cores consume.

The reference product is computed on the CPU, as the reference's harness does with its
rr.ref_gemm (validate.py:29-34): mxfp4_b200.ref dequantises the weight bytes in NumPy and
multiplies in fp32 BLAS, with no GPU code involved, so a dequantisation bug shared by the
kernels and the library's GPU dequantiser cannot pass unseen.  The bit-exact tile check also
compares against that CPU dequantisation.
"""

from __future__ import annotations

import argparse
import logging

import numpy as np
import torch

from . import kernels as kk
from . import ref as cpu_ref

log = logging.getLogger("mxfp4_b200.validate")


def _max_rel_err(out: np.ndarray, ref: np.ndarray, eps: float = 1e-6) -> float:
    return float(np.max(np.abs(out - ref) / np.maximum(np.abs(ref), eps)))


def _bound(out: np.ndarray, ref: np.ndarray) -> float:
    """max|err| / max|ref|, the parity bar of this library (<= 1e-2)."""
    return float(np.max(np.abs(out.astype(np.float64) - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def validate_shape(M: int, N: int, K: int, atol: float = 1e-2, rtol: float = 2e-2) -> bool:
    device = torch.device("cuda:0")
    rng = np.random.default_rng(42)
    A_f32 = rng.standard_normal((M, K), dtype=np.float32) * 0.1
    A = torch.from_numpy(A_f32).to(torch.bfloat16).to(device)
    B_f32 = rng.standard_normal((K, N), dtype=np.float32) * 0.1
    B_packed, B_scales = kk.quantize_mxfp4(torch.from_numpy(B_f32).to(device), axis=0)
    Bp_host, Bs_host = B_packed.cpu().numpy(), B_scales.cpu().numpy()
    C_ref = cpu_ref.ref_gemm(A.float().cpu().numpy(), Bp_host, Bs_host)

    log.info("shape M=%d N=%d K=%d", M, N, K)
    all_ok = True

    def record(label, fn):
        nonlocal all_ok
        try:
            out = fn()
            torch.cuda.synchronize()
            out = out.float().cpu().numpy()
        except RuntimeError as ex:
            log.error("  %s: FAILED %s", label, ex)
            all_ok = False
            return
        ok = bool(np.allclose(out, C_ref, atol=atol, rtol=rtol)) and _bound(out, C_ref) <= 1e-2
        log.info("  %s: max_abs=%.4e max_rel=%.4e bound=%.3e pass=%s", label,
                 float(np.max(np.abs(out - C_ref))), _max_rel_err(out, C_ref), _bound(out, C_ref), ok)
        all_ok = all_ok and ok

    labels = {"A": kk.gemm_a, "B": kk.gemm_b}
    if kk.shape_supported_c(M, N, K):
        labels.update({"C": kk.gemm_c, "D": kk.gemm_d, "E": kk.gemm_e, "F": kk.gemm_f, "H": kk.gemm_h,
                       "I": kk.gemm_i, "K": kk.gemm_k, "J": kk.gemm_j, "M": kk.gemm_m, "AUTO": kk.gemm_auto})
    for label, fn in labels.items():
        record(label, lambda fn=fn: fn(A, B_packed, B_scales))

    if N % 128 == 0 and K % 64 == 0:
        Bp_g, Bs_g = kk.prepack_b_mxfp4(B_packed, B_scales)
        record("G", lambda: kk.gemm_g(A, Bp_g, Bs_g))

    w = kk.prepack_b200(B_packed, B_scales)
    for path in ("tc", "tc_smem", "gemv"):
        if kk.shape_supported(path, M, N, K):
            record(f"b200:{path}", lambda path=path: kk.gemm(A, w, out_dtype=torch.float32, path=path))
    record("b200:bf16-out", lambda: kk.gemm(A, w, out_dtype=torch.bfloat16))

    tile = kk.dequantize_prepacked(w).float().cpu().numpy()  # [N, K]
    ref_tile = np.ascontiguousarray(cpu_ref.dequantize_ref_layout(Bp_host, Bs_host).T)
    exact = bool(np.array_equal(tile, ref_tile))
    log.info("  dequant tile bit-exact=%s", exact)
    all_ok = all_ok and exact
    err = kk.device_error()
    if err:
        log.error("  device error word %d", err)
        all_ok = False
    return all_ok


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="*", default=["256,256,128", "512,512,256", "1024,1024,256"])
    ap.add_argument("--log-level", default="INFO")
    args = ap.parse_args(argv)
    logging.basicConfig(level=args.log_level, format="%(asctime)s %(levelname)s %(name)s: %(message)s")
    ok_all = True
    for s in args.shapes:
        m, n, k = (int(x) for x in s.split(","))
        ok_all = validate_shape(m, n, k) and ok_all
    raise SystemExit(0 if ok_all else 1)


if __name__ == "__main__":
    main()
