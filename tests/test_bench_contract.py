"""bench.py's reference arm on CPU: one JSON line on rank 0 with the GPU arm's workload
record, step and warm-up counts, metric and units; other ranks print nothing."""
from __future__ import annotations

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(rank_env: dict):
    env = dict(os.environ, **rank_env)
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--config", "cfg1", "--steps", "2", "--warmup", "1"],
                         cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    return [line for line in out.stdout.splitlines() if line.strip()]


def test_reference_arm_line_matches_gpu_arm_contract(pkg):
    lines = _run({"RANK": "0", "WORLD_SIZE": "1"})
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "NVFP4 grouped GEMM TFLOP/s (cfg1)"
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["steps"] == 2 and d["warmup"] == 3  # the GPU arm runs max(W, 3) warm-up steps
    assert d["value"] > 0
    # The same workload record the GPU arm prints (built from the same seeded problem).
    sys.path.insert(0, ROOT)
    import bench

    class Args:
        config, experts, split_k = "cfg1", None, False

    prob = pkg.workloads.make_config("cfg1", seed=0, device="cpu")
    assert d["config"] == json.loads(json.dumps(bench.workload_config(Args, prob, 1, False)))
    cpu = d["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == d["value"]
    assert "per step" in cpu["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_runs_on_rank_zero_only():
    assert _run({"RANK": "1", "WORLD_SIZE": "2"}) == []
