"""CPU: the benchmark's measurement contract.

The workloads carry the benchmark configurations' shapes, the algorithmic bytes per step follow the metric's
definition (288 B per attended token row per query group; 1320 B per appended token), the ncu
traffic figures the bench reports are the ones committed in profiles/traffic.json, and the reference
arm (the CPU oracle port, runnable here) prints the one JSON line the driver parses.
"""
import json
import os
import subprocess
import sys

import pytest

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_workloads_carry_the_baseline_shapes():
    w = bench.WORKLOADS
    assert (w["dense8k"]["B"], w["dense8k"]["H"], w["dense8k"]["QL"], w["dense8k"]["ctx"]) == (16, 64, 1, 8192)
    assert (w["sparse"]["B"], w["sparse"]["H"], w["sparse"]["ctx"], w["sparse"]["topk"]) == (16, 64, 131072, 2048)
    assert w["long"]["lens"] == [460000] * 5 + [900000] * 3 and w["long"]["QL"] == 3
    assert (w["append"]["B"], w["append"]["ctx"], w["append"]["pool_tokens"]) == (16, 2048, 2713846)
    assert w["dense128k"]["ctx"] == 131072


def test_algorithmic_bytes_per_step():
    w = bench.WORKLOADS
    assert bench.kv_bytes_per_step(w["dense8k"]) == 16 * 8192 * 288
    assert bench.kv_bytes_per_step(w["dense128k"]) == 16 * 131072 * 288
    assert bench.kv_bytes_per_step(w["sparse"]) == 16 * 2048 * 288
    assert bench.kv_bytes_per_step(w["append"]) == 16 * 2048 * (1024 + 288 + 8)


def test_reported_traffic_comes_from_the_committed_profiles():
    for wl in ("dense8k", "dense128k", "sparse"):
        t = bench.profile_traffic(wl)
        assert t is not None and t > bench.kv_bytes_per_step(bench.WORKLOADS[wl]) * 0.9, wl
    assert bench.profile_traffic("append") > 0
    assert bench.profile_traffic("no-such-workload") is None


@pytest.mark.parametrize("workload", ["dense8k", "append"])
def test_reference_arm_prints_the_contract_line(workload):
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", workload,
                        "--steps", "1", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True,
                       timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["warmup"] >= 3 and line["steps"] == 1 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["higher_is_better"] is True
    assert "workload" in line["config"]
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_under_torchrun_prints_one_line_from_rank_0():
    """The driver launches both arms with torchrun for N > 1: rank 0 alone runs the CPU
    reference and prints; the other ranks exit 0 without work."""
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                        "--master-addr", "127.0.0.1", "--master-port", "29541", "bench.py", "--gpus", "2",
                        "--impl", "reference", "--steps", "1", "--warmup", "1"],
                       cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["n_gpus"] == 2
