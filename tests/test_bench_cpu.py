"""CPU tests of bench.py's host side: the CPU baseline (NumPy port and torch-CPU restatement)
and the reference arm's JSON line, on the small c0 workload."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_cpu_baseline_fields():
    sys.path.insert(0, ROOT)
    import bench

    cb = bench.cpu_baseline("c0", reps=2, rows=64)
    assert cb["kind"] == "port" and cb["unit"] == "TFLOP/s" and cb["value"] > 0
    assert cb["torch_cpu"]["value"] > 0 and cb["torch_cpu"]["threads"] >= 1
    assert cb["cores"] >= 1 and cb["cpu_count"] >= 1 and isinstance(cb["cpu_model"], str)


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "c0",
                        "--steps", "1", "--warmup", "0"], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["metric"] == "c0_tflops" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
    # the reference arm times the workload's full M with every host thread
    assert "M = 128" in line["cpu_baseline"]["sample"] and line["cpu_baseline"]["cores"] == os.cpu_count()


def test_reference_arm_uses_all_threads_under_torchrun_env():
    env = dict(os.environ, OMP_NUM_THREADS="1", WORLD_SIZE="2", RANK="0")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "c0",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"], capture_output=True, text=True,
                       timeout=600, env=env)
    assert r.returncode == 0, r.stderr
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["cpu_baseline"]["cores"] == os.cpu_count() and line["scaling"] == "strong"
    # the other ranks print nothing and exit 0
    env["RANK"] = "1"
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload", "c0",
                        "--gpus", "2", "--steps", "1", "--warmup", "0"], capture_output=True, text=True,
                       timeout=600, env=env)
    assert r.returncode == 0 and r.stdout.strip() == ""
