"""Host parts of bench.py that run without a GPU: the config-1 CPU baseline (the C
restatement of the reference, timed on the host cores) and the argument surface."""

from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import bench
from tests.golden import inputs as I

ROOT = Path(__file__).resolve().parents[1]


def test_decode_cpu_baseline_fields():
    x, w, fp16, int8, n_tr, n_tc = I.config1(0)
    r = bench.decode_cpu_baseline(x, w, fp16, int8, n_tr, n_tc, 9_750_824, seconds=0.1)
    assert r["unit"] == "GB/s" and r["kind"] == "port" and r["cores"] >= 1
    assert r["value"] > 0 and "config-1" in r["sample"]


def test_bench_help_lists_the_workloads():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--help"], capture_output=True, text=True,
                         cwd=ROOT, timeout=300).stdout
    for flag in ("--workload", "--impl", "--tp", "--allreduce", "--gpus", "--steps", "--warmup"):
        assert flag in out
    for workload in ("prefill", "decode", "gemm", "generate"):
        assert workload in out
