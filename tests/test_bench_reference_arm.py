"""CPU tests of `bench.py --impl reference`, the arm the driver times beside
the GPU arm: one JSON line on rank 0 with the GPU arm's metric, unit and
workload, the host cores it really used (torchrun's OMP_NUM_THREADS=1 does
not shrink it), an `e2e` object with no host-device copies, and nothing from
the other ranks.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(extra_env: dict, *args: str) -> subprocess.CompletedProcess:
    env = dict(os.environ)
    env.update(extra_env)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                           "--steps", "1", "--warmup", "0", *args],
                          capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)


def _line(r: subprocess.CompletedProcess) -> dict:
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    return json.loads(lines[0])


def test_single_process_line_follows_the_contract():
    d = _line(_run({"WORLD_SIZE": "1", "RANK": "0"}))
    assert d["impl"] == "reference" and d["metric"] == bench.METRIC
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == bench.CONFIGS["decode"]["desc"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["value"] == d["value"] and cb["cores"] >= 1 and cb["sample"]


def test_under_torchrun_rank0_reports_all_host_cores_and_other_ranks_stay_silent():
    env = {"WORLD_SIZE": "2", "OMP_NUM_THREADS": "1"}
    d = _line(_run(dict(env, RANK="0")))
    assert d["n_gpus"] == 2 and d["scaling"] == "strong"
    assert d["config"]["workload"] == bench.CONFIGS["ep"]["desc"]
    assert d["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0))
    r = _run(dict(env, RANK="1"))
    assert r.returncode == 0 and not r.stdout.strip()
