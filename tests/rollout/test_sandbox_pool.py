"""SandboxPool bookkeeping with fake members (no containers, no git).

Behaviour stated after reference tests/rollout/test_sandbox_pool.py:123-369: a member is created once
and reused after a pristine release; a reset that fails (a mangled container) or a gate that fails
discards it; ``max_uses`` recycles; concurrent acquires get distinct members; ``max_members`` evicts an
idle member of another task, else blocks until a release; a failed setup frees its reserved slot;
``close`` refuses later acquires; ``retire`` hands idle members back. The host-side pristine gate itself
is exercised against real git trees in tests/rollout/test_rollout.py.
"""

from __future__ import annotations

import threading
import time

import pytest

import thundersync_b200.rollout.sandbox_pool as sp
from thundersync_b200.rollout.agent import Task
from thundersync_b200.rollout.sandbox_pool import SandboxPool, SandboxPoolError


class FakeBox:
    def __init__(self, image, name):
        self.image, self.name = image, name
        self.closed = False
        self.pristine = True
        self.mangled = False

    def exec(self, cmd):
        if self.mangled:
            raise RuntimeError("container shell is gone")
        return "TS_POOL_RESET_OK\n"

    def close(self):
        self.closed = True


@pytest.fixture(autouse=True)
def _fake_gate(monkeypatch):
    monkeypatch.setattr(sp, "trusted_tree_pristine", lambda box: box.pristine)


def _pool(**kw):
    return SandboxPool(FakeBox, name_prefix="t", setup=lambda box, task: None, **kw)


A, B = Task("a", "p", "img-a"), Task("b", "p", "img-b")


def test_create_once_then_reuse_and_discard_what_fails_the_gate():
    pool = _pool()
    x = pool.acquire(A)
    pool.release(A, x)
    assert pool.acquire(A) is x and pool.created == 1 and pool.reused == 1
    x.pristine = False
    pool.release(A, x)
    assert x.closed and pool.pristine_failures == 1 and pool.discarded == 1
    y = pool.acquire(A)
    assert y is not x and pool.created == 2
    y.mangled = True
    pool.release(A, y)  # the reset itself failed: discarded, never reused
    assert y.closed and pool.pristine_failures == 2


def test_max_uses_recycles_members():
    pool = _pool(max_uses=2)
    x = pool.acquire(A)
    pool.release(A, x)
    assert pool.acquire(A) is x
    pool.release(A, x)  # second use: expired
    assert x.closed and not pool.pristine_failures
    assert pool.acquire(A) is not x


def test_concurrent_acquires_get_distinct_members_and_close_refuses():
    pool = _pool()
    x, y = pool.acquire(A), pool.acquire(A)
    assert x is not y and pool.report()["members"] == 2
    pool.release(A, x)
    pool.close()
    assert x.closed
    with pytest.raises(SandboxPoolError):
        pool.acquire(A)
    pool.release(A, y)  # a release after close discards
    assert y.closed and pool.report()["members"] == 0


def test_member_cap_evicts_another_tasks_idle_member():
    pool = _pool(max_members=1)
    x = pool.acquire(A)
    pool.release(A, x)
    y = pool.acquire(B)
    assert x.closed and y is not x and pool.evicted == 1 and pool.report()["members"] == 1


def test_member_cap_blocks_until_a_busy_member_is_released():
    pool = _pool(max_members=1)
    x = pool.acquire(A)
    got = {}

    def other():
        got["box"] = pool.acquire(B)

    t = threading.Thread(target=other)
    t.start()
    time.sleep(0.2)
    assert "box" not in got  # blocked: the only member is busy
    pool.release(A, x)
    t.join(timeout=10)
    assert not t.is_alive() and got["box"] is not x and x.closed and pool.evicted == 1


def test_a_failed_setup_frees_its_reserved_slot():
    calls = {"n": 0}

    def setup(box, task):
        calls["n"] += 1
        if calls["n"] == 1:
            raise RuntimeError("image pull failed")

    pool = SandboxPool(FakeBox, name_prefix="t", setup=setup, max_members=1)
    with pytest.raises(RuntimeError):
        pool.acquire(A)
    assert pool.report()["members"] == 0
    x = pool.acquire(A)  # the slot is free again
    assert pool.created == 1 and not x.closed


def test_retire_hands_back_idle_members():
    pool = _pool()
    x = pool.acquire(A)
    pool.release(A, x)
    out = pool.retire()
    assert out == [x] and not x.closed and pool.report()["members"] == 0 and pool.report()["idle"] == 0
