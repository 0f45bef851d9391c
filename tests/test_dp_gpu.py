"""Multi-GPU data parallelism through the native NVLink collectives (2 ranks)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]
ROOT = Path(__file__).resolve().parents[1]


def _run(mode: str, tmp_path, nproc: int = 2) -> dict:
    out = tmp_path / f"{mode}.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=str(ROOT))
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(29600 + hash(mode) % 300),
           str(ROOT / "tests" / "_dp_worker.py"), "--mode", mode, "--out", str(out)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return json.loads(out.read_text())


def test_dp_step_equals_single_process(tmp_path):
    res = _run("equality", tmp_path)
    assert res["path"] == "native", res
    assert res["rel_err"] < 2e-2, res
    assert res["replicas_equal"], res


def test_native_collectives_are_exact_and_deterministic(tmp_path):
    res = _run("native", tmp_path)
    assert res["allreduce_close"] and res["allreduce_bitwise_same"] and res["params_same_after_gather"], res
    assert res["oneshot_equal"], res


def test_device_wait_times_out_with_status(tmp_path):
    res = _run("timeout", tmp_path)
    assert res["status_code"] >= 1000, res


def test_sharded_step_equals_replicated_update(tmp_path):
    """ZeRO-1 over the native collectives: every rank ends with the replicated update's parameters."""
    res = _run("sharded", tmp_path)
    assert res["path"] == "native", res
    assert res["replicas_equal"], res
    assert abs(res["norm"] - res["ref_norm"]) <= 1e-3 * max(1.0, res["ref_norm"]), res
    assert res["max_param_diff"] <= 2e-2, res  # bf16 parameters: at most a rounding apart
