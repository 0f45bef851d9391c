"""Pinned source arena, statistic pools, close-pack profiler (CPU).

Reference behaviour: tests/grpo/test_pinned_arena*.py, test_device_statistics.py
and test_close_profiler.py of the reference: budget formula, smallest-fit
reuse, replacement of too-small free slabs, fail-closed waits, pool misses.
"""

from __future__ import annotations

import json
import threading

import pytest
import torch

from thundersync_b200.grpo.close_profiler import PROFILE_DIR_ENV, ClosePackProfiler
from thundersync_b200.grpo.device_statistics import device_statistic_slots
from thundersync_b200.grpo.pinned_arena import (PinnedSourceArena, PinnedStatisticPool, default_piece_bytes,
                                                host_pinned_budget, tensor_offsets)

PIECE = default_piece_bytes()


def test_budget_and_offsets():
    b, ev = host_pinned_budget(host_ranks=4, host_fraction=0.5, reserved_bytes=10, available_bytes=1000)
    assert b == 1000 * 0.5 // 4 - 10 and ev["rank_share_bytes"] == 125
    offs, total = tensor_offsets([3, 600, 1])
    assert offs == [0, 512, 1536] and total == 1537
    with pytest.raises(ValueError):
        host_pinned_budget(host_ranks=0, host_fraction=0.5, reserved_bytes=0, available_bytes=1)


def test_arena_reuse_replace_and_fail_closed():
    arena = PinnedSourceArena(budget_bytes=3 * PIECE, max_slabs=2)
    a = arena.acquire(PIECE // 2, owner="a", release_possible=lambda: True)
    assert a.capacity == PIECE and a.buffer.numel() == PIECE
    b = arena.try_acquire(PIECE // 4, owner="b")
    assert b is not None and arena.report()["slabs"] == 2
    assert arena.try_acquire(10, owner="c") is None  # cap reached, nothing free
    arena.release(b)
    c = arena.try_acquire(10, owner="c")
    assert c is b  # smallest free slab that fits is reused
    arena.release(a)
    # a 2-piece request: the free 1-piece slab is replaced to fit the budget
    big = arena.try_acquire(PIECE + 1, owner="big")
    assert big is not None and big.capacity == 2 * PIECE and arena.report()["replaced_slabs"] == 1
    with pytest.raises(RuntimeError, match="cannot fold"):
        arena.acquire(PIECE, owner="d", release_possible=lambda: False)
    arena.release(c)
    arena.release(big)
    with pytest.raises(RuntimeError, match="released twice"):
        arena.release(big)
    arena.close()
    with pytest.raises(RuntimeError, match="closed"):
        arena.try_acquire(1, owner="e")


def test_arena_waits_for_release():
    arena = PinnedSourceArena(budget_bytes=PIECE, max_slabs=1)
    a = arena.acquire(100, owner="a", release_possible=lambda: True)
    threading.Timer(0.2, arena.release, args=(a,)).start()
    b = arena.acquire(100, owner="b", release_possible=lambda: True)
    assert b is a and arena.report()["waits"] == 1
    arena.close()


def test_for_host_refuses_below_min_slabs():
    with pytest.raises(RuntimeError, match="holds 0 source slab"):
        PinnedSourceArena.for_host(10 * PIECE, host_ranks=8, host_fraction=0.5, reserved_bytes=0, min_slabs=1,
                                   max_slabs=None, available_bytes=20 * PIECE)
    a = PinnedSourceArena.for_host(PIECE, host_ranks=1, host_fraction=1.0, reserved_bytes=0, min_slabs=1,
                                   max_slabs=None, available_bytes=10 * PIECE)
    assert a.slab_limit == 5  # one slab is 2 pieces (bytes + bytes/32, rounded up)
    with pytest.raises(RuntimeError, match="holds 5"):
        a.extend_slab_limit(1)


def test_statistic_pool_and_slots():
    pool = PinnedStatisticPool([4, 3], torch.float32, slots=1)
    s = pool.acquire("g0")
    assert s is not None and pool.acquire("g1") is None
    v = pool.view(s, 1, torch.Size([3]), statistic="reward")
    v.fill_(2.0)
    assert pool.fits(0, torch.zeros(4)) and not pool.fits(0, torch.zeros(5))
    pool.release(s)
    assert pool.acquire("g2") is s and pool.report()["misses"] == 1
    pool.close()
    assert device_statistic_slots(device_total_bytes=100, parameter_bytes=10, gradient_bytes=10,
                                  optimizer_state_bytes=20, source_bytes=5, device_held_sources=2,
                                  statistic_pair_bytes=8, reserve_bytes=10, open_groups=10) == 5
    assert device_statistic_slots(device_total_bytes=10, parameter_bytes=10, gradient_bytes=10,
                                  optimizer_state_bytes=0, source_bytes=0, device_held_sources=0,
                                  statistic_pair_bytes=8, reserve_bytes=0, open_groups=3) == 0


def test_close_profiler_window(tmp_path, monkeypatch):
    monkeypatch.setenv(PROFILE_DIR_ENV, str(tmp_path))
    monkeypatch.setenv("THUNDERSYNC_GRPO_PROFILE_STEP", "2")
    monkeypatch.setenv("THUNDERSYNC_GRPO_PROFILE_MIN_TOKENS", "5")
    prof = ClosePackProfiler.from_env()
    assert not prof.selects(rank=0, step=1, branch_tokens=[10])
    assert not prof.selects(rank=0, step=2, branch_tokens=[4])
    assert prof.selects(rank=0, step=2, branch_tokens=[10])
    prof.start(rank=0, step=2, trajectory_ids=[7], branch_tokens=[10])
    torch.ones(4).sum()
    prof.stop()
    meta = json.loads((tmp_path / "rank0-step2-pack0.meta.json").read_text())
    assert meta["trajectory_ids"] == [7] and (tmp_path / "rank0-step2-pack0.json.gz").exists()
    assert not prof.selects(rank=0, step=2, branch_tokens=[10])
