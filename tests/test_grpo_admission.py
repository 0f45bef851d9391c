"""GRPO admission policy (FinalFirstAdmission): final work first, then known closes, then content.

Behaviour stated after reference src/thundersync/grpo/admission.py:20-40 and :77-261, checked against a
recording fake trainer: a verdict for a completion not yet prepared turns it into a close (final once
its group's verdicts are all in, known before); final closes ignore the held-source budget, known
closes respect it unless a known reserve is set; a final backlog runs as one forest call once the step
is fully bound; waiting trainer events pause the drain between packs; refusals of bad settings.
"""

from __future__ import annotations

import pytest

from thundersync_b200.grpo.admission import FinalFirstAdmission


class Ledger:
    def __init__(self, held=0, fully_bound=False, known_slabs=None):
        self.calls = []
        self.held = held
        self.fully_bound = fully_bound
        self.known_slabs = known_slabs

    def prepare_trajectories(self, ids):
        self.calls.append(("prepare", tuple(ids)))

    def bind_rewards(self, binds):
        self.calls.append(("bind", tuple(binds)))

    def record_rewards(self, binds):
        self.calls.append(("record", tuple(binds)))

    def close_trajectories(self, closes):
        self.calls.append(("close", tuple(t for t, _ in closes)))

    def close_final_forest(self, closes):
        self.calls.append(("forest", tuple(t for t, _ in closes)))

    def close_group(self, gid):
        self.calls.append(("group", gid))

    def group_reduction_complete(self, gid):
        return True

    def registered_groups_fully_bound(self):
        return self.fully_bound

    def known_slab_capacity(self):
        return self.known_slabs


def _closes(ledger):
    return [c for c in ledger.calls if c[0] in ("close", "forest")]


def _admission(ledger, **kw):
    kw.setdefault("max_held_sources", 2)
    kw.setdefault("in_flight_sources", lambda: ledger.held)
    return FinalFirstAdmission(ledger, group_size=2, max_prepare_pack=1, **kw)


def test_final_closes_run_before_known_and_ignore_the_budget():
    led = Ledger(held=2)  # the held-source budget is full
    adm = _admission(led)
    for g, t in ((0, 1), (1, 10), (1, 11)):
        adm.add_completion(g, t)
    adm.bind_verdict(0, 1, 1.0)  # group 0 has one of two verdicts: known
    adm.bind_verdict(1, 10, 0.0)
    adm.bind_verdict(1, 11, 1.0)  # group 1 complete: both closes final
    assert ("record", ((1, 1.0),)) in led.calls
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (10,)), ("close", (11,))]  # known close 1 waits for the budget
    assert adm.ready_close_backlog == 1
    led.held = 0
    adm.drain_ready_closes()
    assert _closes(led)[-1] == ("close", (1,)) and adm.ready_close_backlog == 0


def test_a_known_close_becomes_final_when_its_group_completes():
    led = Ledger(held=2)
    adm = _admission(led)
    adm.add_completion(0, 1)
    adm.add_completion(0, 2)
    adm.bind_verdict(0, 1, 1.0)
    adm.drain_ready_closes()
    assert _closes(led) == []  # known, budget full
    adm.bind_verdict(0, 2, 0.0)
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (1,)), ("close", (2,))]


def test_known_reserve_runs_known_closes_outside_the_budget():
    led = Ledger(held=2)
    adm = _admission(led, known_reserve_slabs=1)
    for t in (1, 3):
        adm.add_completion(t, t)
    adm.bind_verdict(1, 1, 1.0)
    adm.bind_verdict(3, 3, 0.0)
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (1,))]  # one per drain: the reserve
    led.known_slabs = 0  # the trainer reports no free known slab
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (1,))]
    led.known_slabs = None
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (1,)), ("close", (3,))]


def test_final_backlog_runs_as_one_forest_once_the_step_is_bound():
    led = Ledger(held=0)
    adm = _admission(led, final_forest=True)
    for t in (1, 2):
        adm.add_completion(0, t)
    adm.bind_verdict(0, 1, 1.0)
    adm.bind_verdict(0, 2, 0.0)
    led.fully_bound = True
    adm.drain_ready_closes()
    assert _closes(led) == [("forest", (1, 2))]
    adm.close_ready_groups()
    assert led.calls[-1] == ("group", 0)


def test_waiting_events_pause_the_final_drain_between_packs():
    led = Ledger(held=0)
    events = {"waiting": False}
    adm = _admission(led, events_waiting=lambda: events["waiting"])
    for t in (1, 2):
        adm.add_completion(0, t)
    adm.bind_verdict(0, 1, 1.0)
    adm.bind_verdict(0, 2, 0.0)
    events["waiting"] = True
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (1,))] and adm.ready_close_backlog == 1
    adm.add_completion(5, 50)
    adm.flush_prepares()  # the paused sweep runs no content prepare
    assert ("prepare", (50,)) not in led.calls
    events["waiting"] = False
    adm.drain_ready_closes()
    assert _closes(led) == [("close", (1,)), ("close", (2,))]
    adm.flush_prepares()
    assert led.calls[-1] == ("prepare", (50,))


def test_bad_settings_are_refused():
    led = Ledger()
    with pytest.raises(ValueError):
        FinalFirstAdmission(led, group_size=2, known_reserve_slabs=-1)
    with pytest.raises(ValueError):
        FinalFirstAdmission(led, group_size=2, known_reserve_slabs=1)  # needs a held-source budget
