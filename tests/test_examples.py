"""The shipped examples run end to end (CPU here; the GPU variant on a B200).

Reference behaviour: tests/test_examples.py of the reference (each example
prints one JSON line with a finite, nonzero gradient norm).
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _run(name: str, cuda: bool) -> dict:
    env = dict(os.environ)
    if not cuda:
        env["CUDA_VISIBLE_DEVICES"] = ""
    out = subprocess.run([sys.executable, str(ROOT / "examples" / name)], env=env, capture_output=True, text=True,
                         timeout=600, check=True)
    return json.loads(out.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("name,objective", [("streaming_grpo.py", "grpo"), ("streaming_opd.py", "opd")])
def test_example_cpu(name, objective):
    rec = _run(name, cuda=False)
    assert rec["objective"] == objective and rec["gradient_norm"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("name,objective", [("streaming_grpo.py", "grpo"), ("streaming_opd.py", "opd")])
def test_example_gpu(name, objective):
    rec = _run(name, cuda=True)
    assert rec["objective"] == objective and rec["gradient_norm"] > 0
