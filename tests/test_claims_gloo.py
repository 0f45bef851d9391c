"""Cross-rank work claims over a real TCPStore: four gloo processes race compare-and-set."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_four_processes_claim_each_item_exactly_once(tmp_path):
    out = tmp_path / "claims.json"
    env = dict(os.environ, PYTHONPATH=str(ROOT), CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = ["timeout", "-k", "20", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=4", "--master-addr", "127.0.0.1", "--master-port", "29721",
           str(ROOT / "tests" / "_claims_worker.py"), "--out", str(out)]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    for everyone in json.loads(out.read_text()):
        winners = [item for won in everyone for item in won]
        assert sorted(winners) == list(range(500))  # every item once, none twice
