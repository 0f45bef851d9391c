"""The config-4 (OPD) bench driver: arrival-clock delivery in joint packs under an open-trajectory budget.

The driver is shared by both bench arms, so its delivery rules are part of the benchmark's definition:
every action is delivered exactly once, a trajectory's actions arrive in order and never twice in one
pack, no pack exceeds the pack limit, and at most ``open_budget`` trajectories are open at once.
"""

from __future__ import annotations

import argparse
import importlib.util
import sys
import time
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location("bench_driver_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


class _FakeObjective:
    def __init__(self, seconds_per_action: float) -> None:
        self.delay = seconds_per_action
        self.open: set = set()
        self.max_open = 0
        self.delivered: list = []
        self.pack_sizes: list = []
        self.closed: list = []

    def open_group(self, g, prompt):
        assert g not in self.open
        self.open.add(g)
        self.max_open = max(self.max_open, len(self.open))

    def append_scored_turns(self, items, return_loss):
        assert len({it[1] for it in items}) == len(items), "a trajectory twice in one pack"
        assert len(items) == 1 or sum(len(it[2]) for it in items) <= 1500, "pack over its token limit"
        self.pack_sizes.append(len(items))
        for g, tid, tokens, mask, teacher, weights in items:
            assert g in self.open and len(teacher) == sum(mask)
            self.delivered.append((g, tuple(tokens)))
        time.sleep(self.delay * len(items))

    def close_trajectories(self, ids):
        self.closed.extend(ids)

    def close_group(self, g):
        self.open.discard(g)


@pytest.mark.parametrize("budget,delay", [(None, 0.0), (5, 0.0), (11, 0.002), (11, 0.02)])
def test_opd_driver_delivers_every_action_once_in_order(budget, delay):
    bench = _bench()
    args = argparse.Namespace(seed=3, groups_per_rank=12, prompt_len=4, vocab=50)
    work = bench.make_step_opd(0, 0, args)
    trainer = bench.OPDTrainer.__new__(bench.OPDTrainer)
    trainer.obj = _FakeObjective(delay)
    trainer.device = "cpu"
    trainer.open_budget = budget
    trainer.pack_limit = 4
    trainer.pack_tokens = 1500
    trainer.packs = trainer.packed_actions = 0
    trainer.finish = lambda: {}
    trainer.step_batch(work)
    fake = trainer.obj
    expected: dict = {}
    for ev in work["events"]:
        expected.setdefault(ev[1], []).append(tuple(ev[3]))
    got: dict = {}
    for g, tokens in fake.delivered:
        got.setdefault(g, []).append(tokens)
    assert got == expected
    assert max(fake.pack_sizes) <= 4
    assert sorted(fake.closed) == sorted(expected)
    if budget is not None:
        assert fake.max_open <= budget
