"""Opt-in ``torch.profiler`` window around selected trajectory-close packs (C35).

Enabled by ``THUNDERSYNC_GRPO_PROFILE_DIR``; ``_STEP`` (default 3), ``_RANK``
(0), ``_MIN_TOKENS`` (14000), ``_PACKS`` (1) and ``_STACK`` (``1`` records
Python stacks) under the same ``THUNDERSYNC_GRPO_PROFILE_`` prefix select
which closes are captured. Each window writes
``rank<r>-step<s>-pack<k>.json.gz`` (Chrome trace) and a ``.meta.json``
record (trajectory ids, branch tokens, window seconds). The variable names
and file names are the reference's, so its trace tooling applies
(reference: src/thundersync/grpo/close_profiler.py:27-123).
"""

from __future__ import annotations

import json
import os
import time
from pathlib import Path
from typing import Any

import torch

__all__ = ["ClosePackProfiler", "DEFAULT_PROFILE_MIN_TOKENS", "PROFILE_DIR_ENV"]

PROFILE_DIR_ENV = "THUNDERSYNC_GRPO_PROFILE_DIR"
DEFAULT_PROFILE_MIN_TOKENS = 14000
_PREFIX = "THUNDERSYNC_GRPO_PROFILE_"


def _env_int(suffix: str, default: int) -> int:
    v = os.environ.get(_PREFIX + suffix, "").strip()
    return int(v) if v else default


class ClosePackProfiler:
    def __init__(self, directory: Path, *, step: int, rank: int, min_tokens: int, packs: int,
                 with_stack: bool) -> None:
        self.directory = Path(directory)
        self.step, self.rank = step, rank
        self.min_tokens, self.packs = min_tokens, packs
        self.with_stack = with_stack
        self.taken = 0
        self._prof: Any = None
        self._rec: dict[str, Any] | None = None

    @classmethod
    def from_env(cls) -> "ClosePackProfiler | None":
        d = os.environ.get(PROFILE_DIR_ENV, "").strip()
        if not d:
            return None
        return cls(Path(d), step=_env_int("STEP", 3), rank=_env_int("RANK", 0),
                   min_tokens=_env_int("MIN_TOKENS", DEFAULT_PROFILE_MIN_TOKENS), packs=_env_int("PACKS", 1),
                   with_stack=os.environ.get(_PREFIX + "STACK", "") == "1")

    def selects(self, *, rank: int, step: int, branch_tokens: list[int]) -> bool:
        return (self._prof is None and self.taken < self.packs and rank == self.rank and step == self.step
                and max(branch_tokens, default=0) >= self.min_tokens)

    def start(self, *, rank: int, step: int, trajectory_ids: list[int], branch_tokens: list[int]) -> None:
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
            torch.cuda.synchronize()
        self._prof = torch.profiler.profile(activities=acts, record_shapes=False, with_stack=self.with_stack)
        self._prof.__enter__()
        self._rec = {"rank": rank, "step": step, "pack": self.taken, "trajectory_ids": list(trajectory_ids),
                     "branch_tokens": list(branch_tokens), "started_at": time.perf_counter()}

    def stop(self) -> None:
        prof, rec = self._prof, self._rec
        if prof is None or rec is None:
            return
        self._prof = self._rec = None
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        rec["window_s"] = time.perf_counter() - rec["started_at"]
        prof.__exit__(None, None, None)
        self.directory.mkdir(parents=True, exist_ok=True)
        stem = f"rank{rec['rank']}-step{rec['step']}-pack{rec['pack']}"
        prof.export_chrome_trace(str(self.directory / f"{stem}.json.gz"))
        (self.directory / f"{stem}.meta.json").write_text(json.dumps(rec, indent=2, sort_keys=True) + "\n")
        self.taken += 1
