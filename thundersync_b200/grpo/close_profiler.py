"""Opt-in ``torch.profiler`` capture of selected trajectory-close packs (C35).

Set ``THUNDERSYNC_GRPO_PROFILE_DIR`` to switch it on. Under the same
``THUNDERSYNC_GRPO_PROFILE_`` prefix, ``STEP`` (default 3) and ``RANK`` (0)
pick the step and rank, ``MIN_TOKENS`` (14000) the smallest longest-branch
size worth capturing, ``PACKS`` (1) how many packs to capture, and
``STACK=1`` records Python stacks. Each capture writes a Chrome trace
``rank<r>-step<s>-pack<k>.json.gz`` and a ``.meta.json`` beside it (the
variable names and file names are the interface of reference
src/thundersync/grpo/close_profiler.py:27-123, so trace tooling written for
either package reads both).

The selection rule is a frozen :class:`CaptureRule` read once from the
environment; :class:`ClosePackProfiler` owns the capture budget and at most
one open capture (``selects`` / ``start`` / ``stop``, or ``capture`` as a
context manager).
"""

from __future__ import annotations

import contextlib
import json
import os
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Iterator, Mapping

import torch

__all__ = ["CaptureRule", "ClosePackProfiler", "DEFAULT_PROFILE_MIN_TOKENS", "PROFILE_DIR_ENV"]

PROFILE_DIR_ENV = "THUNDERSYNC_GRPO_PROFILE_DIR"
DEFAULT_PROFILE_MIN_TOKENS = 14000
_VAR = "THUNDERSYNC_GRPO_PROFILE_{}"


@dataclass(frozen=True)
class CaptureRule:
    """Which closes are captured."""

    directory: Path
    step: int = 3
    rank: int = 0
    min_tokens: int = DEFAULT_PROFILE_MIN_TOKENS
    packs: int = 1
    with_stack: bool = False

    @classmethod
    def from_mapping(cls, env: Mapping[str, str]) -> "CaptureRule | None":
        root = env.get(PROFILE_DIR_ENV, "").strip()
        if not root:
            return None

        def number(name: str, fallback: int) -> int:
            raw = env.get(_VAR.format(name), "").strip()
            return int(raw) if raw else fallback

        return cls(Path(root), step=number("STEP", 3), rank=number("RANK", 0),
                   min_tokens=number("MIN_TOKENS", DEFAULT_PROFILE_MIN_TOKENS), packs=number("PACKS", 1),
                   with_stack=env.get(_VAR.format("STACK"), "") == "1")

    def matches(self, *, rank: int, step: int, branch_tokens: list[int]) -> bool:
        return rank == self.rank and step == self.step and max(branch_tokens, default=0) >= self.min_tokens


class ClosePackProfiler:
    """Captures up to ``rule.packs`` close packs that match ``rule``."""

    def __init__(self, directory: Path, *, step: int, rank: int, min_tokens: int, packs: int,
                 with_stack: bool) -> None:
        self.rule = CaptureRule(Path(directory), step=step, rank=rank, min_tokens=min_tokens, packs=packs,
                                with_stack=with_stack)
        self.taken = 0
        self._open: tuple[Any, dict[str, Any]] | None = None

    @classmethod
    def from_env(cls, env: Mapping[str, str] | None = None) -> "ClosePackProfiler | None":
        rule = CaptureRule.from_mapping(os.environ if env is None else env)
        if rule is None:
            return None
        return cls(rule.directory, step=rule.step, rank=rule.rank, min_tokens=rule.min_tokens, packs=rule.packs,
                   with_stack=rule.with_stack)

    @property
    def directory(self) -> Path:
        return self.rule.directory

    def selects(self, *, rank: int, step: int, branch_tokens: list[int]) -> bool:
        """True when a capture should start for this pack (none open, budget left, rule matches)."""
        if self._open is not None or self.taken >= self.rule.packs:
            return False
        return self.rule.matches(rank=rank, step=step, branch_tokens=branch_tokens)

    def start(self, *, rank: int, step: int, trajectory_ids: list[int], branch_tokens: list[int]) -> None:
        activities = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            activities.append(torch.profiler.ProfilerActivity.CUDA)
            torch.cuda.synchronize()  # the window holds this pack's device work only
        session = torch.profiler.profile(activities=activities, record_shapes=False,
                                         with_stack=self.rule.with_stack)
        session.__enter__()
        meta = {"rank": rank, "step": step, "pack": self.taken, "trajectory_ids": list(trajectory_ids),
                "branch_tokens": list(branch_tokens), "t0": time.perf_counter()}
        self._open = (session, meta)

    def stop(self) -> None:
        if self._open is None:
            return
        session, meta = self._open
        self._open = None
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        meta["window_s"] = time.perf_counter() - meta.pop("t0")
        session.__exit__(None, None, None)
        out = self.rule.directory
        out.mkdir(parents=True, exist_ok=True)
        name = "rank{rank}-step{step}-pack{pack}".format(**meta)
        session.export_chrome_trace(str(out / f"{name}.json.gz"))
        (out / f"{name}.meta.json").write_text(json.dumps(meta, indent=2, sort_keys=True) + "\n")
        self.taken += 1

    @contextlib.contextmanager
    def capture(self, *, rank: int, step: int, trajectory_ids: list[int], branch_tokens: list[int]) -> Iterator[bool]:
        """Capture the enclosed close when the rule selects it; yields whether it does."""
        chosen = self.selects(rank=rank, step=step, branch_tokens=branch_tokens)
        if chosen:
            self.start(rank=rank, step=step, trajectory_ids=trajectory_ids, branch_tokens=branch_tokens)
        try:
            yield chosen
        finally:
            if chosen:
                self.stop()
