"""Host parts of bench.py that run without a GPU: the config-1 CPU baseline (the C
restatement of the reference, timed on the host cores) and the argument surface."""

from __future__ import annotations

import os
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


def test_reference_arm_is_host_only():
    """The reference arm times the CPU restatement without this project's GPU library,
    on every host thread even when launched with OMP_NUM_THREADS=1 (as torchrun starts
    each rank)."""
    code = ("import os, sys, types, bench; "
            "a = types.SimpleNamespace(steps=1, warmup=0, cpu_rows=4); "
            "line = bench.run_reference(a, 1, 0); "
            "assert line['impl'] == 'reference' and line['value'] > 0, line; "
            "assert line['config'] == dict(bench.PREFILL_CONFIG, parallelism='one host, all cores'); "
            "assert line['cpu_baseline']['cores'] == (os.cpu_count() or 1), line['cpu_baseline']; "
            "assert 'tilequant_b200' not in sys.modules, 'GPU library imported'; print('ok')")
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=ROOT, timeout=600, env=env)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]
