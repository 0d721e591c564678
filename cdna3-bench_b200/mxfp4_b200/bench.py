"""Per-shape timing sweep of every entry point, written as CSV samples.

    python -m mxfp4_b200.bench [--shapes M,N,K ...] [--out results/sweep.csv]
                               [--warmup 50] [--iters 100]
    python -m mxfp4_b200.bench --quantize [K,N ...]      # GPU quantiser + prepack throughput

Mirrors python/mxfp4_cdna3/bench.py:31-119 (_bench_one, run_sweep): seed-0 inputs
(A ~ N(0,1) bf16, W ~ N(0,1) quantised along K), 8 rotating weight copies, one CUDA event
pair per iteration, p50/p95 and TFLOP/s = 2MNK/p50 per strategy label, and a CSV of
(strategy, M, N, K, iter, ns).  Each row additionally carries the fraction of the shape's
B200 roofline, max(2MNK / P_bf16, weight+scale+activation bytes / BW_hbm), with the peaks
of cost_model.load_peaks.  The reference's violin plot needs matplotlib, which this image
lacks; the CSV holds the same data.
"""

from __future__ import annotations

import argparse
import csv
import logging
from pathlib import Path

import numpy as np
import torch

from . import cost_model as cm
from . import kernels as kk

log = logging.getLogger("mxfp4_b200.bench")


def _alloc_inputs(M: int, N: int, K: int, device):
    gen = torch.Generator(device=device).manual_seed(0)
    A = torch.empty(M, K, dtype=torch.bfloat16, device=device).normal_(0.0, 1.0, generator=gen)
    B = torch.randn(K, N, generator=gen, device=device, dtype=torch.float32)
    B_packed, B_scales = kk.quantize_mxfp4(B, axis=0)
    C = torch.empty(M, N, dtype=torch.float32, device=device)
    return A, B_packed, B_scales, C


def _bench_one(launch_fn, weights, A, C, n_warmup: int, n_iter: int):
    """Event-timed iterations over rotating weight copies; returns ns per iteration."""
    torch.cuda.synchronize()
    for i in range(n_warmup):
        launch_fn(A, weights[i % len(weights)], C)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_iter)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_iter)]
    for i in range(n_iter):
        starts[i].record()
        launch_fn(A, weights[i % len(weights)], C)
        ends[i].record()
    torch.cuda.synchronize()
    return [s.elapsed_time(e) * 1e6 for s, e in zip(starts, ends, strict=True)]


def run_sweep(shapes, out_csv, n_warmup: int = 50, n_iter: int = 100, rot: int = 8):
    device = torch.device("cuda:0")
    peaks = cm.load_peaks()
    rows = []
    for M, N, K in shapes:
        log.info("shape M=%d N=%d K=%d", M, N, K)
        A, B_packed, B_scales, C = _alloc_inputs(M, N, K, device)
        ref_w = [(B_packed.clone(), B_scales.clone()) for _ in range(rot)]
        strategies = {
            "A": (ref_w, lambda a, w, c: kk.gemm_a(a, w[0], w[1], c)),
            "AUTO": (ref_w, lambda a, w, c: kk.gemm_auto(a, w[0], w[1], c)),
        }
        if N % 128 == 0 and K % 64 == 0:
            g_w = [kk.prepack_b_mxfp4(bp, bs) for bp, bs in ref_w]
            strategies["G"] = (g_w, lambda a, w, c: kk.gemm_g(a, w[0], w[1], c))
        pre = [kk.prepack_b200(bp, bs) for bp, bs in ref_w]
        for path in ("tc", "tc_smem", "gemv"):
            if kk.shape_supported(path, M, N, K):
                strategies[f"b200:{path}"] = (pre, lambda a, w, c, p=path: kk.gemm(a, w, torch.float32, p, c))
        roof_us = cm.roofline(cm.Shape(M, N, K), peaks).t_us
        for label, (weights, fn) in strategies.items():
            try:
                ts = _bench_one(fn, weights, A, C, n_warmup, n_iter)
            except RuntimeError as ex:
                log.error("strategy %s FAILED: %s", label, ex)
                continue
            srt = sorted(ts)
            p50, p95 = srt[len(srt) // 2], srt[int(len(srt) * 0.95)]
            log.info("  %s: p50=%.1fus p95=%.1fus %.1fTFLOPS roofline=%.2f", label, p50 / 1e3, p95 / 1e3,
                     2.0 * M * N * K / p50 / 1e3, roof_us * 1e3 / p50)
            for i, t in enumerate(ts):
                rows.append({"strategy": label, "M": M, "N": N, "K": K, "iter": i, "ns": t,
                             "frac_roofline": roof_us * 1e3 / t})
        del A, B_packed, B_scales, C, ref_w, strategies
        torch.cuda.empty_cache()
    out_csv = Path(out_csv)
    out_csv.parent.mkdir(parents=True, exist_ok=True)
    with open(out_csv, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["strategy", "M", "N", "K", "iter", "ns", "frac_roofline"])
        w.writeheader()
        w.writerows(rows)
    log.info("wrote %s (%d samples)", out_csv, len(rows))
    return rows


def bench_quantize(shapes, n_iter: int = 20, rule: str = "ocp") -> list[dict]:
    """GPU quantiser + prepack throughput (the reference does both on the host in NumPy,
    ref.py:14-47 and :85-101).  Bytes = fp32 input read + packed nibbles and scales written,
    and for the prepack the packed weights read + the chunk layout written."""
    dev = torch.device("cuda:0")
    peaks = cm.load_peaks()
    out = []
    for K, N in shapes:
        W = torch.randn(K, N, device=dev) * 0.02
        Bp, Bs = kk.quantize_mxfp4(W, axis=0, rule=rule)
        kk.prepack_b200(Bp, Bs)
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        for _ in range(n_iter):
            kk.quantize_mxfp4(W, axis=0, rule=rule)
        ev[1].record()
        for _ in range(n_iter):
            kk.prepack_b200(Bp, Bs)
        ev[2].record()
        torch.cuda.synchronize()
        tq = ev[0].elapsed_time(ev[1]) / n_iter * 1e3
        tp = ev[1].elapsed_time(ev[2]) / n_iter * 1e3
        qbytes = K * N * 4 + K * N // 2 + K * N // 32
        pbytes = 2 * (K * N // 2 + K * N // 32)
        row = {"K": K, "N": N, "quantize_us": tq, "quantize_gbs": qbytes / tq / 1e3,
               "prepack_us": tp, "prepack_gbs": pbytes / tp / 1e3, "hbm_peak_gbs": peaks.hbm_gbs}
        log.info("quantize %dx%d: %.1f us %.0f GB/s | prepack %.1f us %.0f GB/s (HBM copy peak %.0f)",
                 K, N, tq, row["quantize_gbs"], tp, row["prepack_gbs"], peaks.hbm_gbs)
        out.append(row)
    return out


def summarize(rows) -> dict:
    """(strategy, M, N, K) -> p50 ns, from run_sweep rows."""
    acc: dict = {}
    for r in rows:
        acc.setdefault((r["strategy"], r["M"], r["N"], r["K"]), []).append(r["ns"])
    return {k: float(np.median(v)) for k, v in acc.items()}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", nargs="*", default=["128,3072,3072", "4608,9216,3072", "1,10240,8192"])
    ap.add_argument("--out", default="results/sweep.csv")
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--iters", type=int, default=100)
    ap.add_argument("--quantize", nargs="*", default=None, metavar="K,N",
                    help="time the GPU quantiser and prepack on K x N fp32 weights instead of the GEMM sweep")
    ap.add_argument("--log-level", default="INFO")
    args = ap.parse_args(argv)
    logging.basicConfig(level=args.log_level, format="%(asctime)s %(levelname)s %(name)s: %(message)s")
    if args.quantize is not None:
        bench_quantize([tuple(int(x) for x in s.split(",")) for s in (args.quantize or ["3072,3072", "8192,57344"])])
        return
    shapes = [tuple(int(x) for x in s.split(",")) for s in args.shapes]
    run_sweep(shapes, args.out, args.warmup, args.iters)


if __name__ == "__main__":
    main()
