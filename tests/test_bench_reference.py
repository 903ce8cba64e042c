"""bench.py's reference arm on the CPU (no GPU needed): the line the driver
reads, its keys and units, and the multi-rank behaviour (rank 0 alone
measures and prints; the other ranks exit 0 without work)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _bench(args: list[str], rank: int = 0, world: int = 1) -> subprocess.CompletedProcess:
    env = dict(os.environ, RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world))
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env, capture_output=True,
                          text=True, timeout=240)


REF_ARGS = ["--impl", "reference", "--steps", "2", "--warmup", "1", "--ref-step-seconds", "0.5"]


def test_reference_arm_prints_one_contract_line():
    r = _bench(REF_ARGS + ["--workload", "cfg2"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "TFLOP/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert (d["n_gpus"], d["steps"], d["warmup"]) == (1, 2, 1)
    assert d["config"]["pcp_size"] == 1 and "configs[1]" in d["config"]["workload"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_nothing():
    r = _bench(REF_ARGS + ["--gpus", "2"], rank=1, world=2)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""


def test_reference_arm_rank0_of_two_reports_the_job():
    r = _bench(REF_ARGS + ["--gpus", "2", "--workload", "cfg2"], rank=0, world=2)
    assert r.returncode == 0, r.stderr[-2000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["n_gpus"] == 2 and d["config"]["pcp_size"] == 2


def test_gpu_count_must_match_the_launch():
    r = _bench(REF_ARGS + ["--gpus", "2"], rank=0, world=1)
    assert r.returncode != 0
    assert "WORLD_SIZE" in r.stderr
