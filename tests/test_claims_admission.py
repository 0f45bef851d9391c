"""Cross-rank final-work claims through the GRPO admission (ClaimingFinalFirstAdmission), two ranks as
threads over one in-memory store.

Behaviour stated after reference tests/grpo/test_work_claims_admission.py:328-460: the owner offers its
final closes; an idle peer steals some at the step end; every trajectory runs exactly once (on its owner
or a thief, ceded closes are reported back to the owner's trainer); the owner alone runs everything when
no peer claims; claiming needs the final forest; a thief waiting on a peer that never finishes times out.
"""

from __future__ import annotations

import threading

import pytest

from tests.test_scheduling import DictStore
from thundersync_b200.grpo.claims import ClaimingFinalFirstAdmission, decode_final_work, encode_final_work
from thundersync_b200.scheduling.work_claims import StoreWorkClaims


class Trainer:
    final_forest_max_tokens = 1 << 20

    def __init__(self):
        self.ran, self.ceded, self.claimed, self.calls = [], [], [], []
        self.report = None

    def record_rewards(self, binds):
        pass

    def registered_groups_fully_bound(self):
        return True

    def close_final_forest(self, closes):
        self.ran += [t for t, _ in closes]

    def close_trajectories(self, closes):
        self.ran += [t for t, _ in closes]

    def prepare_trajectories(self, ids):
        self.calls.append(("prepare", tuple(ids)))

    def bind_rewards(self, binds):
        pass

    def close_group(self, gid):
        self.calls.append(("group", gid))

    def group_reduction_complete(self, gid):
        return True

    def final_work(self, tid):
        payload = encode_final_work(group_id=tid // 10, trajectory_id=tid, advantage=0.5, prompt_tokens=[1, 2],
                                    turns=[([3, 4], [True, True])])
        return 4, 10 + tid % 10, payload

    def cede_final_closes(self, closes):
        self.ceded += [t for t, _ in closes]

    def run_claimed_work(self, payloads):
        self.claimed += [decode_final_work(p)[1] for p in payloads]

    def record_work_claims(self, report):
        self.report = report


def _owner_batch(adm, groups):
    for g, tids in groups.items():
        for t in tids:
            adm.add_completion(g, t)
        for t in tids:
            adm.bind_verdict(g, t, float(t % 2))


def _admission(trainer, store, rank, world, **kw):
    claims = StoreWorkClaims(store, rank=rank, world_size=world)
    return ClaimingFinalFirstAdmission(trainer, group_size=4, claims=claims, final_forest=True, poll_s=0.001,
                                       max_held_sources=8, in_flight_sources=lambda: 0, **kw)


def test_every_trajectory_runs_once_and_the_idle_rank_takes_part():
    store = DictStore()
    owner, thief = Trainer(), Trainer()
    a0 = _admission(owner, store, 0, 2)
    a1 = _admission(thief, store, 1, 2)
    groups = {1: [10, 11, 12, 13], 2: [20, 21, 22, 23], 3: [30, 31, 32, 33]}
    _owner_batch(a0, groups)
    a0._offer_final_work()  # rank 0's final closes are on offer before either rank drains

    def idle_rank():
        a1.drain_group_closes()  # nothing of its own: publishes done, then steals until rank 0 is done

    t = threading.Thread(target=idle_rank)
    t.start()
    for _ in range(2000):  # let the idle rank steal before the owner drains (deterministic split)
        if thief.claimed:
            break
        threading.Event().wait(0.005)
    assert thief.claimed, "the idle rank took no work"
    a0.drain_ready_closes()
    a0.close_ready_groups()
    a0.drain_group_closes()
    t.join(timeout=30)
    assert not t.is_alive()
    every = sorted(x for g in groups.values() for x in g)
    assert sorted(owner.ran + thief.claimed) == every
    assert len(set(owner.ran) & set(thief.claimed)) == 0
    assert sorted(owner.ceded) == sorted(thief.claimed)
    assert owner.report is not None and thief.report is not None


def test_the_owner_runs_everything_without_a_peer_claiming():
    store = DictStore()
    owner = Trainer()
    a0 = _admission(owner, store, 0, 1)
    groups = {1: [10, 11, 12, 13]}
    _owner_batch(a0, groups)
    a0.drain_ready_closes()
    a0.close_ready_groups()
    a0.drain_group_closes()
    assert sorted(owner.ran) == [10, 11, 12, 13] and owner.ceded == []


def test_claiming_needs_the_final_forest_and_a_silent_peer_times_out():
    store = DictStore()
    with pytest.raises(ValueError):
        ClaimingFinalFirstAdmission(Trainer(), group_size=4, claims=StoreWorkClaims(store, rank=0, world_size=2),
                                    final_forest=False)
    clock = {"t": 0.0}

    def sleep(s):
        clock["t"] += 1.0

    a1 = _admission(Trainer(), DictStore(), 1, 2, timeout_s=5.0, sleep=sleep, clock=lambda: clock["t"])
    with pytest.raises(RuntimeError, match="did not finish"):
        a1.drain_group_closes()  # rank 0 never publishes done
