"""Data parallelism on CPU: two gloo ranks through torch.distributed.run (the reference's DP modes)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
_PORTS = {"equality": 29711, "unequal": 29712, "broadcast": 29713, "guard": 29714}


def _run(mode: str, tmp_path) -> dict:
    out = tmp_path / f"{mode}.json"
    env = dict(os.environ, PYTHONPATH=str(ROOT), CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="2")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_PORTS[mode]),
           str(ROOT / "tests" / "_dp_cpu_worker.py"), "--mode", mode, "--out", str(out)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.loads(out.read_text())


@pytest.mark.parametrize("mode", ["equality", "unequal"])
def test_dp_reduced_gradient_equals_single_process(mode, tmp_path):
    res = _run(mode, tmp_path)
    assert all(r["rel_err"] < 1e-5 for r in res["ranks"]), res
    assert res["replicas_equal"], res


def test_dp_init_broadcasts_rank0_parameters(tmp_path):
    res = _run("broadcast", tmp_path)
    assert res["replicas_equal"], res


def test_dp_open_group_step_raises_before_any_collective(tmp_path):
    res = _run("guard", tmp_path)
    assert all(r["raised"] for r in res["ranks"]), res
    assert res["replicas_equal"], res
