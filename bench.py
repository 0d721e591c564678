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
* e2e: the same metric through the one-call C-ABI entry mxfp4_gemm (kernels.gemm_packed:
  reference-layout weights, re-laid inside the call into a preallocated workspace) from
  pinned HOST buffers: every step copies activations and weights host->device and the bf16
  outputs device->host inside the timed region.
* roofline: the tensor-core kernel's achieved TFLOP/s (2*M*N*K per launch over its
  CUDA-event duration, events recorded inside the timed region) against the measured peak.
* cpu_baseline: the reference algorithm (NumPy dequant + fp32 BLAS matmul, the oracle port
  of ref.py:75-78) at the workload's full M, on this host's cores.
* extra (N = 1, default workload only): the other measured workloads of the same library on
  the same box -- the chained FLUX block (flux_chain) and the decode shapes at M = 1, 4, 16 --
  each timed the same way with its own roofline fraction.
* N > 1 (torchrun): strong scaling of the same block, column-parallel: every GEMM's N is
  split over the ranks in whole 128-row tiles; each GEMM writes its slice into this GPU's full
  [M, N] output and the copy engines push the slice into every peer's output over NVLink (one
  pitched copy per peer, CUDA IPC buffers) while the next GEMM computes; one stream-ordered
  one-int NCCL all-reduce per step orders the reads; this is the default at 2 GPUs (`--ce`).
  `--fused`, the default at 4 and 8 GPUs, stores every tile into all GPUs' outputs from the GEMM
  epilogue instead; `--unfused` uses an NCCL all-gather per GEMM.  tp_sweep is BASELINE configs[4] in the same form.
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
FLUX_DS = [("qkv", 9216, 3072), ("attn_out", 3072, 3072), ("mlp_up", 12288, 3072), ("mlp_down", 3072, 12288)]
WORKLOADS = {
    "flux_ds": (4608, FLUX_DS),
    "flux_ss": (4608, [("qkv_mlp_up", 21504, 3072), ("out_mlp_down", 3072, 15360)]),
    # the double-stream block's linears chained as in the model (attention itself is out of scope:
    # the Q third of the QKV output stands in for its result), replayed from one CUDA graph
    "flux_chain": (4608, FLUX_DS),
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
TP_MODES = ("fused", "unfused", "ce")  # column-parallel modes (strong scaling)
NVLINK_GBS = 770.0  # measured peer copy per direction on this pool's B200s
EXTRA_WORKLOADS = ("flux_chain", "decode_m1", "decode_m4", "decode_m16")


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="flux_ds", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the extra workloads of the default line")
    ap.add_argument("--mx", choices=["q8", "split2"], default=None,
                    help="block-scaled path (activations coded as E4M3 pieces, kind::mxf8f6f4 MMA; q8: one "
                         "OCP MXFP8 piece, split2: two pieces): one GPU, no e2e or CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--weak", action="store_true",
                    help="N > 1: each rank its own N-slice of a w-times wider layer, no collective (weak scaling)")
    ap.add_argument("--unfused", action="store_true",
                    help="N > 1: GEMM then a separate NCCL all-gather on a second stream")
    ap.add_argument("--fused", action="store_true",
                    help="N > 1 (the default at 4 and 8 GPUs): the all-gather fused into the GEMM epilogue, stores straight into every GPU's "
                         "output over NVLink")
    ap.add_argument("--ce", action="store_true",
                    help="N > 1 (the default at 2 GPUs): each GEMM writes its slice into this GPU's full output and the "
                         "copy engines push it to every peer over NVLink while the next GEMM computes")
    ap.add_argument("--no-graph", action="store_true",
                    help="decode and c0 workloads: launch each GEMM from Python instead of replaying a CUDA graph per step")
    return ap.parse_args(argv)


def is_decode(workload: str) -> bool:
    return workload.startswith("decode")


def unit_scale(workload: str) -> float:
    return 1e9 if is_decode(workload) else 1e12  # GB/s or TFLOP/s


def full_shapes(workload: str):
    return WORKLOADS[workload]


# ----------------------------------------------------------------------------- CPU side
def use_all_host_threads() -> int:
    """Let BLAS and torch use every host core (torchrun sets OMP_NUM_THREADS=1 for its ranks)."""
    n = os.cpu_count() or 1
    try:
        from threadpoolctl import threadpool_limits

        threadpool_limits(limits=n)
    except Exception:
        pass
    try:
        import torch

        torch.set_num_threads(n)
    except Exception:
        pass
    return n


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


def cpu_input(workload: str, gi: int, rows: int | None = None, seed: int = 0):
    """Seeded CPU inputs of GEMM `gi` of the workload at `rows` activation rows (default: the
    workload's full M): (A, B_packed, B_scales, units), units in the metric's base."""
    import numpy as np

    oracle = _oracle()
    M, gemms = full_shapes(workload)
    _, N, K = gemms[gi]
    m = M if rows is None else min(rows, M)
    rng = np.random.default_rng(seed + gi)
    A = rng.standard_normal((m, K), dtype=np.float32)
    W = rng.standard_normal((K, N), dtype=np.float32) * np.float32(0.02)
    Bp, Bs = oracle.quantize_mxfp4_ocp(W, axis=0)
    del W
    units = (N * K // 2 + N * K // 32 + m * K * 2) if is_decode(workload) else 2.0 * m * N * K
    return A, Bp, Bs, units


def time_numpy_port(inp) -> float:
    """Seconds of one call of the reference algorithm (oracle port of ref.py ref_gemm: NumPy
    dequant of the full weights + fp32 BLAS matmul)."""
    oracle = _oracle()
    A, Bp, Bs, _ = inp
    t0 = time.perf_counter()
    oracle.ref_gemm(A, Bp, Bs)
    return time.perf_counter() - t0


def time_torch_port(inp) -> float:
    """Seconds of the torch-CPU restatement: the same NumPy dequant, then torch.matmul in fp32."""
    import torch

    oracle = _oracle()
    A, Bp, Bs, _ = inp
    t0 = time.perf_counter()
    W = torch.from_numpy(oracle.dequantize_mxfp4(Bp, Bs, axis=0))
    torch.matmul(torch.from_numpy(A), W)
    return time.perf_counter() - t0


def cpu_baseline(workload: str, reps: int = 1, rows: int | None = None, gemm_ids=None) -> dict:
    """The CPU baseline of the JSON line: every GEMM of one step at the workload's full M (or
    `rows` rows), the NumPy port (the value) and the torch-CPU restatement, each the median of
    `reps` repetitions of the whole step."""
    import torch

    use_all_host_threads()
    unit = METRICS[workload][1]
    scale = unit_scale(workload)
    M, gemms = full_shapes(workload)
    ids = list(range(len(gemms))) if gemm_ids is None else list(gemm_ids)
    t_np, t_torch, units = [], [], 0.0
    inputs = [cpu_input(workload, gi, rows) for gi in ids]
    units = sum(i[3] for i in inputs)
    for _ in range(reps):
        t_np.append(sum(time_numpy_port(i) for i in inputs))
        t_torch.append(sum(time_torch_port(i) for i in inputs))
    m = M if rows is None else min(rows, M)
    return {"value": units / statistics.median(t_np) / scale, "unit": unit, "cores": cpu_threads(), "kind": "port",
            "sample": f"every GEMM of one {workload} step at M = {m} (the workload's "
                      f"{'full M' if m == M else 'first rows'}): NumPy dequant of the full weights + fp32 BLAS "
                      f"matmul per GEMM (oracle port of ref.py ref_gemm), median of {reps}",
            "torch_cpu": {"value": units / statistics.median(t_torch) / scale, "unit": unit,
                          "threads": torch.get_num_threads(),
                          "sample": f"same GEMMs: NumPy dequant + torch.matmul fp32, median of {reps}"},
            "cpu_count": os.cpu_count(), "cpu_model": cpu_model()}


def run_reference_arm(args, rank: int):
    """The reference's CPU implementation of the path (the oracle port of ref.py ref_gemm:
    NumPy dequant + BLAS matmul with every host thread) on the same config and metric.  Each
    step is one GEMM of the workload at its full M, round robin over the workload's GEMMs (the
    dequant of that GEMM's weights happens inside the call, as in the reference).  Under
    torchrun only rank 0 runs it."""
    if rank != 0:
        return
    cores = use_all_host_threads()
    metric, unit = METRICS[args.workload]
    M, gemms = full_shapes(args.workload)
    inputs = {}

    def inp(i):
        gi = i % len(gemms)
        if gi not in inputs:
            inputs[gi] = cpu_input(args.workload, gi)
        return inputs[gi]

    for i in range(args.warmup):
        time_numpy_port(inp(i))
    units, secs = 0.0, 0.0
    for i in range(args.steps):
        x = inp(i)
        secs += time_numpy_port(x)
        units += x[3]
    value = units / secs / unit_scale(args.workload)
    sample = (f"one {args.workload} GEMM per step at the full M = {M} (round robin over {len(gemms)} GEMMs): "
              "NumPy dequant of that GEMM's weights + fp32 BLAS matmul, as ref.py ref_gemm does per call")
    print(json.dumps({
        "impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": secs / max(1, args.steps) * 1e3,
        "higher_is_better": True, "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded N(0,1) activations, N(0,0.02) OCP-MXFP4 weights)",
        "config": {"workload": args.workload, "M": M, "gemms": gemms},
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": sample,
                         "cpu_model": cpu_model(), "blas_threads": cpu_threads()},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, index: int, period_s: float = 0.001):
        self.index, self.period = index, period_s
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._started = threading.Event()
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
            self._started.set()
            time.sleep(self.period)

    def __enter__(self):
        if self.nv is not None:
            self._thr = threading.Thread(target=self._run, daemon=True)
            self._thr.start()
            self._started.wait(1.0)
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
class Ctx:
    """Process-group facts and helpers shared by the measurements."""

    def __init__(self):
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            import datetime

            # a rank that stops early makes the others fail within minutes instead of waiting in
            # a collective for the default ten
            dist.init_process_group("nccl", device_id=self.dev, timeout=datetime.timedelta(seconds=180))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())


def tp_mode(args, ctx, workload: str) -> str:
    """How the workload runs on this job: 'single' (one GPU), 'weak' (each rank its own slice of
    a w-times wider layer), 'fused' / 'unfused' (column-parallel, all-gather fused or NCCL)."""
    if ctx.world == 1:
        return "single"
    if args.weak and workload != "tp_sweep":
        return "weak"
    if args.unfused:
        return "unfused"
    if args.fused:
        return "fused"
    if args.ce:
        return "ce"
    # Measured on B200 (20 steps, flux_ds): the copy-engine push leads at 2 GPUs (1907 vs 1880
    # TFLOP/s), the fused epilogue at 4 (1945 vs 1712) and 8 (1694 vs 1306).
    return "fused" if ctx.world >= 4 else "ce"


def measure(args, ctx, workload: str, steps: int, warmup: int, want_e2e: bool) -> dict:
    """Time `steps` steps of `workload` (after `warmup`) and return the numbers of its line."""
    import torch

    import mxfp4_b200 as mx
    from mxfp4_b200 import cost_model
    from mxfp4_b200 import kernels as kk
    from mxfp4_b200 import sharding

    world, rank, dev = ctx.world, ctx.rank, ctx.dev
    mode = tp_mode(args, ctx, workload)
    M, full = full_shapes(workload)
    decode = is_decode(workload)
    scale = unit_scale(workload)
    chain = workload == "flux_chain"
    if chain and mode != "single":
        raise SystemExit("flux_chain runs on one GPU")

    # this rank's GEMMs: its column slice (tp), or the full layer (single / weak: every rank
    # computes its own slice of a w-times wider layer, i.e. the full per-rank shape)
    gemms = []
    for name, N, K in full:
        if mode in TP_MODES:
            n0, n1 = sharding.column_slice(N, world, rank)
            gemms.append((name, N, n0, n1 - n0, K))
        else:
            gemms.append((name, N, 0, N, K))

    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    items = []
    for name, N_full, n0, N, K in gemms:
        A = torch.randn((M, K), generator=gen, device=dev).to(torch.bfloat16)
        W = torch.randn((K, N), generator=gen, device=dev) * 0.02
        Bp, Bs = mx.quantize_mxfp4(W, axis=0, rule="ocp")
        del W
        items.append({"name": name, "N": N, "N_full": N_full, "n0": n0, "K": K, "A": A, "Bp": Bp, "Bs": Bs,
                      "w": mx.prepack_b200(Bp, Bs), "wmx": kk.prepack_mx(Bp, Bs) if args.mx else None,
                      "C": torch.empty((M, N), dtype=torch.bfloat16, device=dev)})
    # work units of the whole job per step (strong scaling: the full layer once; otherwise each
    # rank's own work, summed over ranks)
    flops_rank = sum(2.0 * M * it["N"] * it["K"] for it in items)
    bytes_rank = sum(cost_model.Shape(M, it["N"], it["K"]).in_bytes for it in items)
    if mode in TP_MODES:
        units_job = sum(cost_model.Shape(M, N, K).in_bytes if decode else 2.0 * M * N * K for _, N, K in full)
    else:
        units_job = world * (bytes_rank if decode else flops_rank)

    # decode and c0 weights fit in L2: rotate copies so the bytes between two reads of one copy
    # exceed L2 (c0's activations, 0.8 MB, stay resident as they would in a serving loop)
    small = decode or workload == "c0"
    rot = 1
    if small:
        l2 = torch.cuda.get_device_properties(dev).L2_cache_size
        rot = max(1, -(-3 * l2 // bytes_rank))
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

    peer = None
    comm = torch.cuda.Stream(dev) if mode == "unfused" else None
    gathered = [None] * len(items)
    if mode in ("fused", "ce"):
        peer = [sharding.PeerOutput(M, it["N_full"], torch.bfloat16) for it in items]
    ce_streams = [torch.cuda.Stream(dev) for _ in range(world - 1)] if mode == "ce" else None
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in items]
          for _ in range(steps)]

    def step(i_step: int, record: bool):
        for j, it in enumerate(items):
            w = it["w_rot"][i_step % rot] if small else (it["wmx"] if args.mx else it["w"])
            if record:
                ev[i_step][j][0].record()
            if mode == "fused":
                kk.gemm_allgather(it["A"], w, peer[j].ptrs, it["n0"], it["N_full"])
            elif mode == "ce":
                kk.gemm_allgather(it["A"], w, [peer[j].ptrs[rank]], it["n0"], it["N_full"])
            else:
                run_gemm(it, w)
            if record:
                ev[i_step][j][1].record()
            if mode == "unfused":
                # the all-gather of this GEMM's slice runs on its own stream while the next GEMM
                # computes (the block's four GEMMs are independent)
                done = torch.cuda.Event()
                done.record()
                comm.wait_event(done)
                with torch.cuda.stream(comm):
                    gathered[j] = sharding.all_gather_columns(it["C"], it["N_full"])
            if mode == "ce":
                # the copy engines push this slice to every peer (one stream per peer) while the
                # next GEMM computes
                done = torch.cuda.Event()
                done.record()
                for cs in ce_streams:
                    cs.wait_event(done)
                peer[j].push(it["n0"], it["n0"] + it["N"], ce_streams)
        if mode == "ce":
            for cs in ce_streams:
                torch.cuda.current_stream().wait_stream(cs)
        if mode in ("fused", "ce"):  # one stream-ordered collective: every peer's stores have landed
            peer[-1].sync()
        if mode == "unfused":  # the step ends when every gather has landed
            torch.cuda.current_stream().wait_stream(comm)

    for i in range(warmup):
        step(i, False)
    ctx.barrier()

    # Decode and c0 GEMMs last ~5-60 us, about the host cost of a Python launch: a serving loop
    # replays them from a CUDA graph, and so does the bench (one graph per weight rotation,
    # with timing events recorded as graph nodes around every GEMM).
    graphs = None
    if chain:
        # h -> QKV -> (Q third as the attention stand-in) -> attn_out -> h + . -> MLP-up -> GELU
        # (tanh) -> MLP-down -> h + .   Only the four GEMMs count as work; the torch
        # element-wise ops between them are inside the timed graph.
        from mxfp4_b200.flux import FluxChain

        fc = FluxChain([it["w"] for it in items], items[0]["A"])
        gev = [[(torch.cuda.Event(enable_timing=True, external=True),
                 torch.cuda.Event(enable_timing=True, external=True)) for _ in items]]
        for _ in range(2):
            fc.forward(gev[0])
        torch.cuda.synchronize()
        gch = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gch):
            fc.forward(gev[0])
        graphs = [gch]
        gch.replay()
        ctx.barrier()

        def step(i_step: int, record: bool):  # noqa: F811
            gch.replay()
    elif small and not args.no_graph and mode in ("single", "weak"):
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
        ctx.barrier()

        def step(i_step: int, record: bool):  # noqa: F811
            graphs[i_step % rot].replay()

    sampler = ClockSampler(ctx.local)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        ctx.barrier()
        t0.record()
        for i in range(steps):
            step(i, True)
        t1.record()
        ctx.barrier()
    total_ms = t0.elapsed_time(t1)
    assert mx.device_error() == 0, "a kernel recorded a device error"
    if graphs is None:
        launch_ms = [statistics.mean(ev[i][j][0].elapsed_time(ev[i][j][1]) for i in range(steps))
                     for j in range(len(items))]
    else:  # each graph's events hold its last replay inside the timed region
        launch_ms = [statistics.mean(gev[r][j][0].elapsed_time(gev[r][j][1]) for r in range(min(len(gev), steps)))
                     for j in range(len(items))]
    ms_step = ctx.max_over_ranks(total_ms / steps)
    launch_ms = [ctx.max_over_ranks(x) for x in launch_ms]
    value = units_job / (ms_step * 1e-3) / scale

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
        ach = bytes_rank / (sum(launch_ms) * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": peaks.hbm_gbs, "unit": "GB/s",
                "frac": ach / peaks.hbm_gbs,
                "kernel": "quant_act_mx8_kernel + gemv_mx_kernel (+ finalize)" if args.mx else "gemv_kernel",
                "peak_source": f"{peaks.source} hbm_gbs (copy)"}
    elif args.mx:  # 8-bit MMA: no fp8 GEMM is measured on this pool; its nominal rate is twice bf16
        ach = flops_rank / (sum(launch_ms) * 1e-3) / 1e12
        pk = 2.0 * (peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops)
        roof = {"bound": "tensor", "achieved": ach, "peak": pk, "unit": "TFLOP/s", "frac": ach / pk,
                "kernel": "quant_act_mx8_kernel + gemm_mx_kernel",
                "peak_source": f"2 x {peaks.source} {'sustained' if sustained else 'burst'} cuBLAS bf16 "
                               "(the 8-bit MMA rate is twice the 16-bit one)"}
    else:
        ach = flops_rank / (sum(launch_ms) * 1e-3) / 1e12
        pk = peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops
        roof = {"bound": "tensor", "achieved": ach, "peak": pk, "unit": "TFLOP/s", "frac": ach / pk,
                "kernel": "gemm_tc_kernel",
                "peak_source": f"{peaks.source} {'sustained' if sustained else 'burst'} cuBLAS bf16"}
    roof["traffic"] = None if (args.mx or mode != "single") else load_traffic(workload)
    nvlink = None
    if mode in TP_MODES:
        # every GPU sends its slice of every output to each peer and receives the rest
        sent = sum(M * it["N"] * 2 * (world - 1) for it in items)
        recv = sum(M * (N - it["N"]) * 2 for it, (_, N, _) in zip(items, full))
        link = max(sent, recv)
        t_link = link / (NVLINK_GBS * 1e9)
        t_comp = flops_rank / ((peaks.bf16_tflops_sustained if sustained else peaks.bf16_tflops) * 1e12)
        nvlink = {"bytes_sent_per_gpu": sent, "bytes_received_per_gpu": recv,
                  "achieved_gbs": link / (ms_step * 1e-3) / 1e9, "peak_gbs": NVLINK_GBS,
                  "frac": link / (ms_step * 1e-3) / 1e9 / NVLINK_GBS,
                  "t_link_us": t_link * 1e6, "t_compute_us": t_comp * 1e6,
                  "bound": "nvlink" if t_link > t_comp else "compute",
                  "step_roofline_frac": max(t_link, t_comp) / (ms_step * 1e-3)}
        if mode == "fused" and t_link > t_comp:
            ach = link / (sum(launch_ms) * 1e-3) / 1e9
            roof = {"bound": "nvlink", "achieved": ach, "peak": NVLINK_GBS, "unit": "GB/s",
                    "frac": ach / NVLINK_GBS, "kernel": "gemm_tc_kernel (all-gather epilogue)",
                    "peak_source": "measured NVLink peer copy per direction", "traffic": None}

    e2e = None
    if want_e2e and mode == "single" and not chain and not args.mx:
        e2e = run_e2e(args, ctx, mx, items, M, units_job, scale, METRICS[workload][1], warmup, steps)

    # our kernels per step: the GEMM, plus the decode activation prestage (4 <= M <= 16) or the
    # split-K reduction (small M x N) where the workspace plan has them; the block-scaled path
    # adds its activation coder (and, for decode, the bf16 conversion)
    if args.mx:
        per_step = len(items) * (3 if decode else 2)
    elif mode in ("fused", "ce"):
        per_step = len(items)
    else:
        per_step = sum(1 + (mx.workspace_bytes(M, it["N"], it["K"], "prepacked") > 0 and M >= 4) for it in items)
    launches = steps * per_step
    return {"workload": workload, "mode": mode, "M": M, "items": items, "value": value, "ms_step": ms_step,
            "per_gemm": per_gemm, "roofline": roof, "nvlink": nvlink, "e2e": e2e, "rot": rot, "small": small,
            "graphs": graphs is not None, "chain": chain, "bytes_rank": bytes_rank, "launches": launches,
            "clocks": sampler.summary(), "total_ms": total_ms}


def parallelism_text(mode: str, world: int) -> str:
    return {"single": "one GPU",
            "weak": f"weak x{world}: each rank its own N-slice of a {world}x wider layer, no collective",
            "fused": f"tp{world} column-parallel, all-gather fused into the GEMM epilogue (NVLink stores into every "
                     "GPU's full output)",
            "ce": f"tp{world} column-parallel, local GEMM into the full output + copy-engine push of the slice "
                  "to every peer over NVLink (overlapped with the next GEMM)",
            "unfused": f"tp{world} column-parallel, local GEMM + NCCL all-gather (each gather overlapped with "
                       "the next GEMM on a second stream)"}[mode]


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank)
        return

    import torch

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    ctx = Ctx()
    metric, unit = METRICS[args.workload]
    if args.mx:
        if args.workload in ("flux_chain", "tp_sweep") or world > 1:
            raise SystemExit("--mx: flux_ds, flux_ss, c0 or decode_* on one GPU")
        metric, args.no_e2e, args.no_cpu_baseline = f"{metric}_mx_{args.mx}", True, True

    r = measure(args, ctx, args.workload, args.steps, args.warmup, not args.no_e2e)
    M = r["M"]
    per_rank = [[it["name"], it["N"], it["K"]] for it in r["items"]]
    out_bytes = sum(M * it["N"] * 2 for it in r["items"])

    extra = None
    if (world == 1 and args.workload == "flux_ds" and not args.mx and not args.no_extra):
        extra = {}
        for wl in EXTRA_WORKLOADS:
            del_items(r)
            x = measure(args, ctx, wl, min(args.steps, 20), max(3, args.warmup), False)
            m, u = METRICS[wl]
            extra[wl] = {"metric": m, "value": x["value"], "unit": u, "ms_per_step": x["ms_step"],
                         "roofline_frac": x["roofline"]["frac"], "roofline_kernel": x["roofline"]["kernel"],
                         "per_gemm": {k: {"us": v["us"], "frac_of_roofline": v["frac_of_roofline"],
                                          "hbm_gbs" if is_decode(wl) else "tflops":
                                          v["hbm_gbs"] if is_decode(wl) else v["tflops"]}
                                      for k, v in x["per_gemm"].items()},
                         "launch": "one CUDA graph per step", "clocks": x["clocks"],
                         "l2": (f"{x['rot']} rotating weight copies (> 3x L2 per pass)" if x["small"]
                                else "inputs larger than L2")}
            del_items(x)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload, reps=1)

    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": r["value"], "unit": unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_step"], "higher_is_better": True,
            "scaling": "strong" if r["mode"] in TP_MODES else "weak", "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 activations, N(0,0.02) OCP-MXFP4 weights)",
            "config": {
                "workload": args.workload, "M": M,
                "gemms": [[n, N, K] for n, N, K in full_shapes(args.workload)[1]],
                "gemms_per_rank": per_rank,
                "weights": "MXFP4 (E2M1 + E8M0/32), prepacked, resident in HBM",
                "activations": (f"coded inside each step as E4M3 pieces + E8M0/32 ({args.mx}), block-scaled MMA"
                                if args.mx else "bf16"),
                "output": "bf16", "accumulate": "fp32",
                "l2": (f"{r['rot']} rotating weight copies (> 3x L2 per pass)" if r["small"]
                       else "inputs larger than L2: one step touches "
                            f"{(r['bytes_rank'] + out_bytes) / 1e6:.0f} MB per GPU"),
                "launch": "one CUDA graph per step" if r["graphs"] else "eager, one launch per GEMM",
                "chain": ("QKV -> Q third (attention stand-in) -> attn_out -> residual -> MLP-up -> GELU(tanh) "
                          "-> MLP-down -> residual; torch element-wise ops inside the timed graph") if r["chain"] else None,
                "parallelism": parallelism_text(r["mode"], world),
            },
            "roofline": r["roofline"], "per_gemm": r["per_gemm"], "nvlink": r["nvlink"], "e2e": r["e2e"],
            "cpu_baseline": cpu, "extra": extra, "gpu_launches": r["launches"], "clocks": r["clocks"],
        }), flush=True)
    if world > 1:
        ctx.dist.destroy_process_group()


def del_items(r: dict):
    """Free a measurement's device buffers before the next one allocates its own."""
    import torch

    r.get("items", []).clear()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def run_e2e(args, ctx, mx, items, M, units_step, scale, unit, warmup, steps):
    """The same step through the public one-call entry (kernels.gemm_packed -> mxfp4_gemm with
    the reference layout and a preallocated workspace) from pinned host buffers.  Per GEMM:
    the weights and the activations go host->device, the GEMM re-lays the weights and
    multiplies, the bf16 output comes back; the activations and outputs move in 256-row-tile
    chunks on three streams (upload / compute / download) so the copies overlap the GEMMs."""
    import torch

    from mxfp4_b200 import kernels as kk

    dev = ctx.dev
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
        ws = torch.empty(kk.workspace_bytes(M, it["N"], it["K"], "ref"), dtype=torch.uint8, device=dev)
        devb.append((torch.empty_like(it["A"]), torch.empty_like(it["Bp"]), torch.empty_like(it["Bs"]),
                     torch.empty_like(it["C"]), ws))
        h2d += hA.numel() * 2 + hBp.numel() + hBs.numel()
        d2h += hC.numel() * hC.element_size()
    s_in, s_cmp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)

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
                e_a = []
                for r in range(n_chunks):
                    dA[bounds[r]:bounds[r + 1]].copy_(hA[bounds[r]:bounds[r + 1]], non_blocking=True)
                    e_a.append(torch.cuda.Event())
                    e_a[-1].record(s_in)
            for r in range(n_chunks):
                s_cmp.wait_event(e_a[r])
                with torch.cuda.stream(s_cmp):
                    # one call: re-lay the reference-layout weights into the workspace and multiply
                    kk.gemm_packed(dA[bounds[r]:bounds[r + 1]], dBp, dBs, C=dC[bounds[r]:bounds[r + 1]],
                                   workspace=ws)
                    e_c = torch.cuda.Event()
                    e_c.record(s_cmp)
                s_out.wait_event(e_c)
                with torch.cuda.stream(s_out):
                    hC[bounds[r]:bounds[r + 1]].copy_(dC[bounds[r]:bounds[r + 1]], non_blocking=True)
        end.record(s_out)
        end.synchronize()  # the host reads the step's result
        return start.elapsed_time(end)

    for _ in range(max(1, warmup)):
        e2e_step()
    ctx.barrier()
    n = max(3, min(steps, 20))
    ms = ctx.max_over_ranks(statistics.mean(e2e_step() for _ in range(n)))
    return {"value": units_step / (ms * 1e-3) / scale, "unit": unit,
            "ms_per_step": ms, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": n,
            "path": "public one-call API kernels.gemm_packed (C ABI mxfp4_gemm, reference-layout weights re-laid "
                    "inside each call into a preallocated workspace) from pinned host buffers: weights and "
                    "activations uploaded, output downloaded every step, in 256-row-tile chunks on 3 streams "
                    "(H2D / compute / D2H) overlapped"}


if __name__ == "__main__":
    main()
