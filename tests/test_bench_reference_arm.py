"""The bench's reference arm on the CPU: `bench.py --impl reference` times the reference's
routed-expert path (the NumPy port of experts.py:82-110) on the host cores and prints one
JSON line with the same metric, unit and config as the B200 arm. Under torchrun only rank 0
works and prints; the other ranks exit 0 without output."""

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(*extra, env_extra=None):
    env = dict(os.environ)
    for name in ("RANK", "WORLD_SIZE", "LOCAL_RANK"):
        env.pop(name, None)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *extra],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    import bench

    proc = _run("--steps", "2", "--warmup", "3", "--ref-budget", "0.3")
    assert proc.returncode == 0, proc.stderr[-2000:]
    lines = [l for l in proc.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, proc.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "GB/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["steps"] == 2 and line["warmup"] == 3
    assert line["config"]["workload"] == "expert_gemm_q6_k_m16"
    assert line["config"]["experts_per_gpu"] == bench.EXPERTS
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["unit"] == "GB/s"
    assert line["value"] > 0 and base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_exit_quietly():
    proc = _run("--steps", "1", "--warmup", "3", "--ref-budget", "0.1",
                env_extra={"RANK": "1", "WORLD_SIZE": "2", "LOCAL_RANK": "1"})
    assert proc.returncode == 0, proc.stderr[-2000:]
    assert proc.stdout.strip() == ""


@pytest.mark.parametrize("impl", ["reference", "b200"])
def test_bench_refuses_fewer_than_three_warmup_steps(impl):
    proc = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", impl, "--warmup", "2"],
                          cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert proc.returncode == 2 and "--warmup must be >= 3" in proc.stderr
