#!/usr/bin/env python
"""Benchmark of the MXFP4 x BF16 GEMM library on B200 (driver contract: one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload flux_ds|flux_ss|flux_chain|c0|
                     decode_m1|decode_m4|decode_m16|tp_sweep] [--impl ours|reference]

Default workload = BASELINE configs[1]: one FLUX.1-dev double-stream block's four linears
at M = 4608 tokens (QKV 9216x3072, attn-out 3072x3072, MLP-up 12288x3072, MLP-down
3072x12288), bf16 activations ~ N(0,1), weights ~ N(0,0.02) OCP-MXFP4-quantised along K,
bf16 output, fp32 accumulation.  One step = the four GEMMs.  Synthetic, seeded data.

* value: whole-job TFLOP/s with inputs resident in HBM (prepacked weights), device-timed
  with CUDA events between barriers, max over ranks.  A step touches ~510 MB (> 126 MB L2),
  so each step's inputs have left L2 before the next step reads them.
* e2e: the same metric through the one-call C-ABI entry (weights in the reference layout,
  re-laid inside the call) with pinned HOST buffers: every step copies activations and
  weights host->device and the bf16 outputs device->host inside the timed region.
* roofline: the tensor-core kernel's achieved TFLOP/s (2*M*N*K per launch over its
  CUDA-event duration, events recorded inside the timed region) against the measured peak.
* cpu_baseline: the reference algorithm (NumPy dequant + fp32 BLAS matmul, the oracle port
  of ref.py:75-78) on a bounded sample of the workload, on this host's cores.
* N > 1 (torchrun, NCCL): each rank owns its own N-slice of a w-times wider layer and runs
  the same per-rank block (weak scaling, no collective on the data path); tp_sweep is the
  strong-scaling column-parallel config with an NCCL all-gather of the output.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "cdna3-bench_b200"))

DECODE = [("qkv", 10240, 8192), ("o_proj", 8192, 8192), ("gate_up", 57344, 8192), ("down", 8192, 28672)]
WORKLOADS = {
    "flux_ds": (4608, [("qkv", 9216, 3072), ("attn_out", 3072, 3072), ("mlp_up", 12288, 3072),
                       ("mlp_down", 3072, 12288)]),
    "flux_ss": (4608, [("qkv_mlp_up", 21504, 3072), ("out_mlp_down", 3072, 15360)]),
    # the double-stream block's linears chained as in the model (attention itself is out of scope:
    # the Q third of the QKV output stands in for its result), replayed from one CUDA graph
    "flux_chain": (4608, [("qkv", 9216, 3072), ("attn_out", 3072, 3072), ("mlp_up", 12288, 3072),
                          ("mlp_down", 3072, 12288)]),
    "c0": (128, [("c0", 3072, 3072)]),
    "decode_m1": (1, DECODE),
    "decode_m4": (4, DECODE),
    "decode_m16": (16, DECODE),
    "tp_sweep": (8192, [("gate_up", 57344, 8192)]),
}
METRICS = {
    "flux_ds": ("flux_ds_block_tflops", "TFLOP/s"),
    "flux_ss": ("flux_ss_block_tflops", "TFLOP/s"),
    "flux_chain": ("flux_chain_block_tflops", "TFLOP/s"),
    "c0": ("c0_tflops", "TFLOP/s"),
    "decode_m1": ("decode_m1_hbm_gbs", "GB/s"),
    "decode_m4": ("decode_m4_hbm_gbs", "GB/s"),
    "decode_m16": ("decode_m16_hbm_gbs", "GB/s"),
    "tp_sweep": ("tp_sweep_tflops", "TFLOP/s"),
}
REF_SAMPLE_ROWS = 256  # activation rows per GEMM in the CPU samples


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="flux_ds", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--mx", choices=["q8", "split2"], default=None,
                    help="block-scaled path (activations coded as E4M3 pieces, kind::mxf8f6f4 MMA; q8: one "
                         "OCP MXFP8 piece, split2: two pieces): one GPU, no e2e or CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--allgather", action="store_true", help="all-gather outputs (column-parallel)")
    ap.add_argument("--unfused", action="store_true",
                    help="column-parallel: GEMM then a separate NCCL all-gather (default: all-gather fused "
                         "into the GEMM epilogue, stores straight into every GPU's output over NVLink)")
    ap.add_argument("--no-graph", action="store_true",
                    help="decode and c0 workloads: launch each GEMM from Python instead of replaying a CUDA graph per step")
    return ap.parse_args()


def shapes_for(workload: str, world: int):
    M, gemms = WORKLOADS[workload]
    if workload == "tp_sweep":  # strong scaling: the fixed layer is split column-wise
        from mxfp4_b200.sharding import column_slice

        rank = int(os.environ.get("RANK", "0"))
        out = []
        for n, N, K in gemms:
            n0, n1 = column_slice(N, world, rank)
            out.append((n, n1 - n0, K))
        return M, out
    return M, gemms


def is_decode(workload: str) -> bool:
    return workload.startswith("decode")


def unit_scale(workload: str) -> float:
    return 1e9 if is_decode(workload) else 1e12  # GB/s or TFLOP/s


# ----------------------------------------------------------------------------- CPU side
def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info

        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        if n:
            return int(max(n))
    except Exception:
        pass
    return os.cpu_count() or 1


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


def _oracle():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import mxfp4_ref as oracle

    return oracle


def cpu_inputs(workload: str, gemm_ids, rows: int, seed: int = 0):
    """Seeded CPU inputs for `rows` activation rows of each listed GEMM of the workload:
    [(A, B_packed, B_scales, units)] with units in the metric's base (FLOP or bytes)."""
    import numpy as np

    oracle = _oracle()
    M, gemms = shapes_for(workload, 1)
    rng = np.random.default_rng(seed)
    out = []
    for gi in gemm_ids:
        _, N, K = gemms[gi]
        m = min(rows, M)
        A = rng.standard_normal((m, K), dtype=np.float32)
        W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(0.02)
        Bp, Bs = oracle.quantize_mxfp4_ocp(W, axis=0)
        del W
        units = (N * K // 2 + N * K // 32 + m * K * 2) if is_decode(workload) else 2.0 * m * N * K
        out.append((A, Bp, Bs, units))
    return out


def time_numpy_port(inputs) -> float:
    """Seconds of the reference algorithm (oracle port of ref.py ref_gemm: NumPy dequant of the
    full weights + fp32 BLAS matmul) over the inputs."""
    oracle = _oracle()
    secs = 0.0
    for A, Bp, Bs, _ in inputs:
        t0 = time.perf_counter()
        oracle.ref_gemm(A, Bp, Bs)
        secs += time.perf_counter() - t0
    return secs


def time_torch_port(inputs) -> float:
    """Seconds of the torch-CPU restatement: the same NumPy dequant, then torch.matmul in fp32."""
    import torch

    oracle = _oracle()
    secs = 0.0
    for A, Bp, Bs, _ in inputs:
        t0 = time.perf_counter()
        W = torch.from_numpy(oracle.dequantize_mxfp4(Bp, Bs, axis=0))
        torch.matmul(torch.from_numpy(A), W)
        secs += time.perf_counter() - t0
    return secs


def cpu_sample(workload: str, gemm_ids, rows: int, seed: int = 0):
    """Time the reference CPU algorithm (oracle port of ref.py ref_gemm) on `rows` activation
    rows of each listed GEMM; returns (units, seconds) in the metric's unit base."""
    inputs = cpu_inputs(workload, gemm_ids, rows, seed)
    return sum(u for *_, u in inputs), time_numpy_port(inputs)


def cpu_baseline(workload: str, n_gemms: int, rows: int, reps: int = 3) -> dict:
    """The CPU baseline of the JSON line: the NumPy port (the value) and the torch-CPU
    restatement, each the median of `reps` timed repetitions on the same bounded sample."""
    import statistics as st

    import torch

    unit = METRICS[workload][1]
    scale = unit_scale(workload)
    inputs = cpu_inputs(workload, list(range(n_gemms)), rows)
    units = sum(u for *_, u in inputs)
    t_np = st.median(time_numpy_port(inputs) for _ in range(reps))
    t_torch = st.median(time_torch_port(inputs) for _ in range(reps))
    M = shapes_for(workload, 1)[0]
    return {"value": units / t_np / scale, "unit": unit, "cores": cpu_threads(), "kind": "port",
            "sample": f"{min(rows, M)} activation rows of each GEMM of the step: NumPy dequant of the full "
                      f"weights + fp32 BLAS matmul (oracle port of ref.py), median of {reps}",
            "torch_cpu": {"value": units / t_torch / scale, "unit": unit, "threads": torch.get_num_threads(),
                          "sample": "same sample: NumPy dequant + torch.matmul fp32, median of "
                                    f"{reps}"},
            "cpu_count": os.cpu_count(), "cpu_model": cpu_model()}


def run_reference_arm(args, rank: int):
    """The reference's CPU implementation of the path (the oracle port: NumPy + BLAS with every
    host thread) on the same config and metric, one bounded sample per step."""
    if rank != 0:
        return
    metric, unit = METRICS[args.workload]
    n_gemm = len(shapes_for(args.workload, 1)[1])
    for i in range(args.warmup):
        cpu_sample(args.workload, [i % n_gemm], REF_SAMPLE_ROWS, seed=i)
    units, secs = 0.0, 0.0
    for i in range(args.steps):
        u, s = cpu_sample(args.workload, [i % n_gemm], REF_SAMPLE_ROWS, seed=100 + i)
        units += u
        secs += s
    value = units / secs / unit_scale(args.workload)
    M, gemms = shapes_for(args.workload, 1)
    sample = (f"{REF_SAMPLE_ROWS} activation rows of one {args.workload} GEMM per step (round robin): "
              "full NumPy dequant of that GEMM's weights + fp32 BLAS matmul")
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02) OCP-MXFP4 weights)",
        "config": {"workload": args.workload, "M": M, "gemms": gemms},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cpu_threads(), "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period_s: float = 0.005):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thr = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nv = None

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thr:
            self._thr.join()

    def summary(self):
        if self.nv is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"]}
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [n for b, n in self.REASONS.items() if self.reasons & b]}


def load_traffic(workload: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        return json.load(f).get(workload)


# ----------------------------------------------------------------------------- GPU side
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import torch
    import torch.distributed as dist

    import mxfp4_b200 as mx
    from mxfp4_b200 import kernels as kk
    from mxfp4_b200 import cost_model

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    metric, unit = METRICS[args.workload]
    if args.mx:
        if args.workload in ("flux_chain", "tp_sweep") or world > 1:
            raise SystemExit("--mx: flux_ds, flux_ss, c0 or decode_* on one GPU")
        metric, args.no_e2e, args.no_cpu_baseline = f"{metric}_mx_{args.mx}", True, True
    M, gemms = shapes_for(args.workload, world)
    decode = is_decode(args.workload)
    scale = unit_scale(args.workload)

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)  # each rank: its own weight slice
    items = []
    for name, N, K in gemms:
        A = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        W = torch.randn((K, N), generator=gen, device=dev) * 0.02
        Bp, Bs = mx.quantize_mxfp4(W, axis=0, rule="ocp")
        del W
        items.append({"name": name, "N": N, "K": K, "A": A, "Bp": Bp, "Bs": Bs,
                      "w": mx.prepack_b200(Bp, Bs), "wmx": kk.prepack_mx(Bp, Bs) if args.mx else None,
                      "C": torch.empty((M, N), dtype=torch.bfloat16, device=dev)})
    flops_step = sum(2.0 * M * it["N"] * it["K"] for it in items)
    bytes_step = sum(cost_model.Shape(M, it["N"], it["K"]).in_bytes for it in items)
    units_step = bytes_step if decode else flops_step

    # decode and c0 weights fit in L2: rotate copies so the bytes between two reads of one copy
    # exceed L2 (c0's activations, 0.8 MB, stay resident as they would in a serving loop)
    small = decode or args.workload == "c0"
    rot = 1
    if small:
        l2 = torch.cuda.get_device_properties(dev).L2_cache_size
        rot = max(1, -(-3 * l2 // bytes_step))
        for it in items:
            it["w_rot"] = [it["w"]] + [mx.MXFP4Weight(it["w"].data.clone(), it["w"].N, it["w"].K)
                                       for _ in range(rot - 1)]
            if args.mx:
                it["w_rot"] = [it["wmx"]] + [kk.MXWeight(it["wmx"].data.clone(), it["N"], it["K"])
                                             for _ in range(rot - 1)]

    def run_gemm(it, w):
        """One GEMM of the step on the selected path (w: the weights in that path's layout)."""
        if args.mx:
            return kk.gemm_mx(it["A"], w, mode=args.mx, C=it["C"])
        return mx.gemm(it["A"], w, C=it["C"])

    gather = fused = None
    if world > 1 and (args.allgather or args.workload == "tp_sweep"):
        from mxfp4_b200.sharding import all_gather_columns

        full_n = [N for _, N, _ in WORKLOADS[args.workload][1]] if args.workload == "tp_sweep" \
            else [world * it["N"] for it in items]
        gather = lambda j, Y: all_gather_columns(Y, full_n[j])  # noqa: E731
        fused = None
        if not args.unfused:
            from mxfp4_b200 import sharding

            fused = [sharding.PeerOutput(M, full_n[j], torch.bfloat16) for j in range(len(items))]
            offs = [sharding.column_slice(full_n[j], world, rank)[0] if args.workload == "tp_sweep"
                    else rank * it["N"] for j, it in enumerate(items)]

    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in items]
          for _ in range(args.steps)]

    def step(i_step: int, record: bool):
        for j, it in enumerate(items):
            w = it["w_rot"][i_step % rot] if small else (it["wmx"] if args.mx else it["w"])
            if record:
                ev[i_step][j][0].record()
            if fused is not None:
                kk.gemm_allgather(it["A"], w, fused[j].ptrs, offs[j], fused[j].N)
            else:
                run_gemm(it, w)
            if record:
                ev[i_step][j][1].record()
            if fused is not None:
                fused[j].sync()
            elif gather is not None:
                gather(j, it["C"])

    for i in range(args.warmup):
        step(i, False)
    barrier()

    # Decode and c0 GEMMs last ~5-60 us, about the host cost of a Python launch: a serving loop
    # replays them from a CUDA graph, and so does the bench (one graph per weight rotation,
    # with timing events recorded as graph nodes around every GEMM).
    graphs = None
    chain = args.workload == "flux_chain"
    if chain:
        # h -> QKV -> (Q third as the attention stand-in) -> attn_out -> h + . -> MLP-up -> GELU
        # (tanh) -> MLP-down -> h + .   Only the four GEMMs count as work; the torch
        # element-wise ops between them are inside the timed graph.
        import torch.nn.functional as F

        x0 = items[0]["A"]
        attn_in = torch.empty((M, 3072), dtype=torch.bfloat16, device=dev)
        h = torch.empty_like(x0)
        out = torch.empty_like(x0)
        gev = [[(torch.cuda.Event(enable_timing=True, external=True),
                 torch.cuda.Event(enable_timing=True, external=True)) for _ in items]]

        def chain_body():
            def g(j, a):
                gev[0][j][0].record()
                y = mx.gemm(a, items[j]["w"], C=items[j]["C"])
                gev[0][j][1].record()
                return y

            qkv = g(0, x0)
            attn_in.copy_(qkv[:, :3072])
            h.copy_(x0).add_(g(1, attn_in))
            act = F.gelu(g(2, h), approximate="tanh")
            torch.add(h, g(3, act), out=out)

        for _ in range(2):
            chain_body()
        torch.cuda.synchronize()
        gch = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gch):
            chain_body()
        graphs = [gch]
        gch.replay()
        barrier()

        def step(i_step: int, record: bool):  # noqa: F811
            gch.replay()
    elif small and not args.no_graph and gather is None:
        graphs, gev = [], []
        for r in range(rot):
            evs = [(torch.cuda.Event(enable_timing=True, external=True),
                    torch.cuda.Event(enable_timing=True, external=True)) for _ in items]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for j, it in enumerate(items):
                    evs[j][0].record()
                    run_gemm(it, it["w_rot"][r])
                    evs[j][1].record()
            graphs.append(g)
            gev.append(evs)
        for r in range(rot):
            graphs[r].replay()
        barrier()

        def step(i_step: int, record: bool):  # noqa: F811
            graphs[i_step % rot].replay()

    sampler = ClockSampler(local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        barrier()
        t0.record()
        for i in range(args.steps):
            step(i, True)
        t1.record()
        barrier()
    total_ms = t0.elapsed_time(t1)
    assert mx.device_error() == 0, "a kernel recorded a device error"
    if graphs is None:
        launch_ms = [statistics.mean(ev[i][j][0].elapsed_time(ev[i][j][1]) for i in range(args.steps))
                     for j in range(len(items))]
    else:  # each graph's events hold its last replay inside the timed region
        launch_ms = [statistics.mean(gev[r][j][0].elapsed_time(gev[r][j][1]) for r in range(min(len(gev), args.steps)))
                     for j in range(len(items))]
    ms_step = max_over_ranks(total_ms / args.steps)
    value = world * units_step / (ms_step * 1e-3) / scale

    peaks = cost_model.load_peaks()
    sustained = total_ms > 1000.0
    per_gemm = {}
    for it, lm in zip(items, launch_ms):
        sh = cost_model.Shape(M, it["N"], it["K"])
        rl = cost_model.roofline(sh, peaks, sustained)
        per_gemm[it["name"]] = {"M": M, "N": it["N"], "K": it["K"], "us": lm * 1e3,
                                "tflops": sh.flops / (lm * 1e-3) / 1e12,
                                "hbm_gbs": sh.in_bytes / (lm * 1e-3) / 1e9,
                                "roofline_us": rl.t_us, "frac_of_roofline": rl.t_us / (lm * 1e3),
                                "bound": rl.bound}
    if decode:
        ach = bytes_step / (sum(launch_ms) * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": peaks.hbm_gbs, "unit": "GB/s",
                "frac": ach / peaks.hbm_gbs, "kernel": "gemv_kernel",
                "peak_source": f"{peaks.source} hbm_gbs (copy)"}
    elif args.mx and decode:
        ach = bytes_step / (sum(launch_ms) * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": peaks.hbm_gbs, "unit": "GB/s",
                "frac": ach / peaks.hbm_gbs, "kernel": "quant_act_mx8_kernel + gemv_mx_kernel (+ finalize)",
                "peak_source": f"{peaks.source} hbm_gbs (copy)"}
    elif args.mx:  # 8-bit MMA: no fp8 GEMM is measured on this pool; its nominal rate is twice bf16
        ach = flops_step / (sum(launch_ms) * 1e-3) / 1e12
        pk = 2.0 * (peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops)
        roof = {"bound": "tensor", "achieved": ach, "peak": pk, "unit": "TFLOP/s", "frac": ach / pk,
                "kernel": "quant_act_mx8_kernel + gemm_mx_kernel",
                "peak_source": f"2 x {peaks.source} {'sustained' if sustained else 'burst'} cuBLAS bf16 "
                               "(the 8-bit MMA rate is twice the 16-bit one)"}
    else:
        ach = flops_step / (sum(launch_ms) * 1e-3) / 1e12
        pk = peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops
        roof = {"bound": "tensor", "achieved": ach, "peak": pk, "unit": "TFLOP/s", "frac": ach / pk,
                "kernel": "gemm_tc_kernel",
                "peak_source": f"{peaks.source} {'sustained' if sustained else 'burst'} cuBLAS bf16"}
    roof["traffic"] = None if args.mx else load_traffic(args.workload)
    if fused is not None:  # the fused GEMM + all-gather: compute or NVLink, whichever is slower
        link_gbs = 770.0  # measured peer copy per direction on this pool's B200s
        sent = sum(M * it["N"] * 2 * (world - 1) for it in items)
        t_link = sent / (link_gbs * 1e9)
        t_comp = flops_step / (peaks.bf16_tflops_sustained * 1e12)
        if t_link > t_comp:
            ach = sent / (sum(launch_ms) * 1e-3) / 1e9
            roof = {"bound": "nvlink", "achieved": ach, "peak": link_gbs, "unit": "GB/s", "frac": ach / link_gbs,
                    "kernel": "gemm_tc_kernel (all-gather epilogue)",
                    "peak_source": "measured NVLink peer copy per direction", "traffic": None}

    e2e = None
    if not args.no_e2e and args.workload not in ("tp_sweep", "flux_chain"):
        e2e = run_e2e(args, mx, items, M, dev, units_step, scale, max_over_ranks, barrier, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload, len(items), 4 * REF_SAMPLE_ROWS, reps=1 if decode else 3)

    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": value, "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong" if args.workload == "tp_sweep" else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 activations, N(0,0.02) OCP-MXFP4 weights)",
            "config": {
                "workload": args.workload, "M": M,
                "gemms": [[it["name"], it["N"], it["K"]] for it in items],
                "weights": "MXFP4 (E2M1 + E8M0/32), prepacked, resident in HBM",
                "activations": (f"coded inside each step as E4M3 pieces + E8M0/32 ({args.mx}), block-scaled MMA"
                                if args.mx else "bf16"),
                "output": "bf16", "accumulate": "fp32",
                "l2": (f"{rot} rotating weight copies (> 3x L2 per pass)" if small
                       else "inputs larger than L2: one step touches "
                            f"{(bytes_step + sum(M * it['N'] * 2 for it in items)) / 1e6:.0f} MB"),
                "launch": "one CUDA graph per step" if graphs is not None else "eager, one launch per GEMM",
                "chain": ("QKV -> Q third (attention stand-in) -> attn_out -> residual -> MLP-up -> GELU(tanh) "
                          "-> MLP-down -> residual; torch element-wise ops inside the timed graph") if chain else None,
                "parallelism": (f"tp{world} column-parallel, all-gather fused into the GEMM epilogue (NVLink "
                                "stores into every GPU's output)" if fused is not None else
                                f"tp{world} column-parallel + NCCL all-gather" if gather is not None
                                else f"weak x{world}, per-rank N-slice, no collective"),
            },
            "roofline": roof, "per_gemm": per_gemm, "e2e": e2e, "cpu_baseline": cpu,
            "gpu_launches": args.steps * sum((3 if decode else 2) if args.mx
                                             else 1 + (mx.workspace_bytes(M, it["N"], it["K"], "prepacked") > 0)
                                             for it in items), "clocks": sampler.summary(),
        }), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, mx, items, M, dev, units_step, scale, max_over_ranks, barrier, world):
    import torch

    h2d = d2h = 0
    host, devb = [], []
    for it in items:
        hA = torch.empty(it["A"].shape, dtype=torch.bfloat16, pin_memory=True)
        hA.copy_(it["A"])
        hBp = torch.empty(it["Bp"].shape, dtype=torch.uint8, pin_memory=True)
        hBp.copy_(it["Bp"])
        hBs = torch.empty(it["Bs"].shape, dtype=torch.uint8, pin_memory=True)
        hBs.copy_(it["Bs"])
        hC = torch.empty(it["C"].shape, dtype=it["C"].dtype, pin_memory=True)
        host.append((hA, hBp, hBs, hC))
        ws = torch.empty(mx.workspace_bytes(M, it["N"], it["K"]), dtype=torch.uint8, device=dev)
        devb.append((torch.empty_like(it["A"]), torch.empty_like(it["Bp"]), torch.empty_like(it["Bs"]),
                     torch.empty_like(it["C"]), ws))
        h2d += hA.numel() * 2 + hBp.numel() + hBs.numel()
        d2h += hC.numel() * hC.element_size()
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

    # Row chunks of whole 256-row tiles: compute on chunk r overlaps the upload of chunk r+1 and
    # the download of chunk r-1 (weights go first; they are re-laid once per GEMM).
    tiles = -(-M // 256)
    n_chunks = max(1, min(3, tiles))
    bounds = [min(M, (tiles * r // n_chunks) * 256) for r in range(n_chunks + 1)]

    def e2e_step():
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(s_in)
        for (hA, hBp, hBs, hC), (dA, dBp, dBs, dC, ws) in zip(host, devb):
            with torch.cuda.stream(s_in):
                dBp.copy_(hBp, non_blocking=True)
                dBs.copy_(hBs, non_blocking=True)
                e_w = torch.cuda.Event()
                e_w.record(s_in)
                e_a = []
                for r in range(n_chunks):
                    dA[bounds[r]:bounds[r + 1]].copy_(hA[bounds[r]:bounds[r + 1]], non_blocking=True)
                    e_a.append(torch.cuda.Event())
                    e_a[-1].record(s_in)
            s_cmp.wait_event(e_w)
            with torch.cuda.stream(s_cmp):
                w = mx.prepack_b200(dBp, dBs)
            for r in range(n_chunks):
                s_cmp.wait_event(e_a[r])
                with torch.cuda.stream(s_cmp):
                    mx.gemm(dA[bounds[r]:bounds[r + 1]], w, C=dC[bounds[r]:bounds[r + 1]])
                    e_c = torch.cuda.Event()
                    e_c.record(s_cmp)
                s_out.wait_event(e_c)
                with torch.cuda.stream(s_out):
                    hC[bounds[r]:bounds[r + 1]].copy_(dC[bounds[r]:bounds[r + 1]], non_blocking=True)
        end.record(s_out)
        end.synchronize()  # the host reads the step's result
        return start.elapsed_time(end)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    barrier()
    n = max(3, min(args.steps, 20))
    ms = max_over_ranks(statistics.mean(e2e_step() for _ in range(n)))
    return {"value": world * units_step / (ms * 1e-3) / scale, "unit": METRICS[args.workload][1],
            "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": n,
            "path": "public API from pinned host buffers: reference-layout weights uploaded and re-laid "
                    "(prepack_b200) once per GEMM, activations uploaded, multiplied (gemm) and downloaded "
                    "in 256-row-tile chunks, 3 streams (H2D / compute / D2H) overlapped"}


if __name__ == "__main__":
    main()
