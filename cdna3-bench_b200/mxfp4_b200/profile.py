"""Profiling helpers: a one-shape driver to run under ncu, and summaries of ncu output.

    # run one entry point `--iters` times (wrap the command in ncu)
    python -m mxfp4_b200.profile one --path tc --M 4608 --N 9216 --K 3072
    # summarise a launch list (ncu --metrics gpu__time_duration.sum --clock-control none --csv --log-file L.csv)
    python -m mxfp4_b200.profile launches L.csv
    # summarise a capture (ncu -i R.ncu-rep --page raw --csv > R.csv)
    python -m mxfp4_b200.profile raw R.csv

Mirrors python/mxfp4_cdna3/profile_one.py:13-71 (seeded inputs, one strategy, --iters calls)
and profile_summary.py:41-165 (per-kernel duration table with shares, counter summary); the
counters are ncu's instead of rocprof's: tensor-pipe activity for the large-M kernel, DRAM
bytes and throughput for the decode kernel, issue and ALU activity for both.
"""

from __future__ import annotations

import argparse
import csv
import io
import statistics
import sys
from collections import defaultdict

# ncu raw-page metrics worth reading for these kernels (name -> label)
KEY_METRICS = {
    "gpu__time_duration.sum": "duration",
    "dram__bytes_read.sum": "DRAM read",
    "dram__bytes_write.sum": "DRAM write",
    "gpu__dram_throughput.avg.pct_of_peak_sustained_elapsed": "DRAM throughput % of peak",
    "sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active": "tensor pipe % active",
    "smsp__issue_active.avg.pct_of_peak_sustained_active": "issue active %",
    "sm__inst_executed_pipe_alu.avg.pct_of_peak_sustained_active": "ALU pipe %",
    "sm__warps_active.avg.pct_of_peak_sustained_active": "warps active %",
    "launch__registers_per_thread": "registers / thread",
    "launch__grid_size": "grid size",
    "lts__t_sector_hit_rate.pct": "L2 hit rate %",
}


def short_name(name: str) -> str:
    """Kernel name without arguments, e.g. 'void mxb::gemv_kernel<1, bf16>(...)' -> 'mxb::gemv_kernel<1, bf16>'."""
    n = name.strip().strip('"')
    if n.startswith("void "):
        n = n[5:]
    depth, out = 0, []
    for ch in n:
        if ch == "(" and depth == 0:
            break
        depth += ch == "<"
        depth -= ch == ">"
        out.append(ch)
    return "".join(out).strip()


def _table_rows(text: str):
    """Rows of an ncu CSV, skipping the '==PROF==' preamble ncu may write before the header."""
    lines = [ln for ln in text.splitlines() if ln and not ln.startswith("==")]
    return list(csv.reader(io.StringIO("\n".join(lines))))


def parse_launches(text: str) -> dict[str, list[float]]:
    """ncu launch list (--metrics gpu__time_duration.sum --csv) -> kernel -> durations in ns."""
    rows = _table_rows(text)
    if not rows:
        return {}
    h = rows[0]
    kn, mn, mu, mv = (h.index("Kernel Name"), h.index("Metric Name"), h.index("Metric Unit"), h.index("Metric Value"))
    scale = {"ns": 1.0, "nsecond": 1.0, "us": 1e3, "usecond": 1e3, "ms": 1e6, "msecond": 1e6}
    out: dict[str, list[float]] = defaultdict(list)
    for r in rows[1:]:
        if len(r) <= mv or r[mn] != "gpu__time_duration.sum":
            continue
        out[short_name(r[kn])].append(float(r[mv].replace(",", "")) * scale.get(r[mu], 1.0))
    return dict(out)


def launch_table(durs: dict[str, list[float]]) -> str:
    total = sum(sum(v) for v in durs.values()) or 1.0
    lines = ["| kernel | launches | total µs | p50 µs | share |", "|---|---|---|---|---|"]
    for k, v in sorted(durs.items(), key=lambda kv: -sum(kv[1])):
        name = k if len(k) <= 80 else k[:77] + "..."
        lines.append(f"| {name} | {len(v)} | {sum(v) / 1e3:.1f} | {statistics.median(v) / 1e3:.1f} | "
                     f"{100.0 * sum(v) / total:.1f} % |")
    return "\n".join(lines)


def parse_raw(text: str) -> list[dict[str, str]]:
    """`ncu -i rep --page raw --csv` -> one {metric: 'value unit'} dict per captured launch."""
    rows = _table_rows(text)
    if len(rows) < 3:
        return []
    h, units = rows[0], rows[1]
    out = []
    for r in rows[2:]:
        d = {}
        for i, k in enumerate(h):
            if i < len(r):
                d[k] = f"{r[i]} {units[i]}".strip() if i < len(units) else r[i]
        out.append(d)
    return out


def raw_table(launch: dict[str, str]) -> str:
    name = short_name(launch.get("Kernel Name", "?"))
    lines = [f"kernel: {name}", "", "| metric | value |", "|---|---|"]
    for k, label in KEY_METRICS.items():
        if k in launch:
            lines.append(f"| {label} (`{k}`) | {launch[k]} |")
    return "\n".join(lines)


def run_one(path: str, M: int, N: int, K: int, iters: int, seed: int) -> None:
    """Seeded inputs (A, W ~ 0.1*N(0,1), reference quantisation) and `iters` calls of one path."""
    import numpy as np
    import torch

    from . import kernels as kk

    dev = torch.device("cuda:0")
    rng = np.random.default_rng(seed)
    A = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32) * 0.1).to(torch.bfloat16).to(dev)
    W = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * 0.1).to(dev)
    Bp, Bs = kk.quantize_mxfp4(W, axis=0)
    if path in ("tc", "tc_smem", "gemv", "auto"):
        w = kk.prepack_b200(Bp, Bs)
        C = torch.empty((M, N), dtype=torch.bfloat16, device=dev)

        def call():
            kk.gemm(A, w, C=C, path=path)
    elif path == "g":
        gp, gs = kk.prepack_b_mxfp4(Bp, Bs)
        C = torch.empty((M, N), dtype=torch.float32, device=dev)

        def call():
            kk.gemm_g(A, gp, gs, C)
    else:
        fn = getattr(kk, f"gemm_{path}")
        C = torch.empty((M, N), dtype=torch.float32, device=dev)

        def call():
            fn(A, Bp, Bs, C)
    for _ in range(iters):
        call()
    torch.cuda.synchronize()
    print(f"{path} M={M} N={N} K={K} iters={iters}")


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    one = sub.add_parser("one")
    one.add_argument("--path", default="auto",
                     choices=["auto", "tc", "tc_smem", "gemv", "a", "b", "c", "d", "e", "f", "g", "h", "i", "j", "k", "m"])
    one.add_argument("--M", type=int, required=True)
    one.add_argument("--N", type=int, required=True)
    one.add_argument("--K", type=int, required=True)
    one.add_argument("--iters", type=int, default=10)
    one.add_argument("--seed", type=int, default=0)
    la = sub.add_parser("launches")
    la.add_argument("csv")
    rw = sub.add_parser("raw")
    rw.add_argument("csv")
    args = ap.parse_args(argv)
    if args.cmd == "one":
        run_one(args.path, args.M, args.N, args.K, args.iters, args.seed)
    elif args.cmd == "launches":
        with open(args.csv) as f:
            print(launch_table(parse_launches(f.read())))
    else:
        with open(args.csv) as f:
            for launch in parse_raw(f.read()):
                print(raw_table(launch))
                print()


if __name__ == "__main__":
    main(sys.argv[1:])
