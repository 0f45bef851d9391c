"""GRPO admission: final work first, then known closes, then content (C43, GRPO policy).

A verdict for a completion that is still waiting to be prepared records the
reward in the trainer's ledger and makes the trajectory a close. The close is
*final* when every verdict of its group has landed (its advantage is then
fixed) and *known* otherwise. ``drain_ready_closes`` runs final closes first
and outside the residency budget, then known closes within it; with
``final_forest`` a backlog that is all final once the step's last verdict
landed runs as one shared-prefix forest call; with ``known_reserve_slabs``
known closes run outside the held-source budget, up to the reserve per drain.
Between packs the admission yields to waiting trainer events
(``events_waiting``). The policy is that of
reference src/thundersync/grpo/admission.py:77-261; the code is this
package's: closes are ranked by a class function and drained class by class.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable
from typing import Any, Protocol

from thundersync_b200.scheduling.admission import (Close, CloseCoefficient, ContentReadyAdmission, EarlyTrainer,
                                                   TrainerCall, direct_call)

__all__ = ["GroupLedgerTrainer", "FinalFirstAdmission"]


class GroupLedgerTrainer(EarlyTrainer, Protocol):
    def record_rewards(self, binds: list[tuple[int, CloseCoefficient]]) -> None: ...
    def registered_groups_fully_bound(self) -> bool: ...
    def close_final_forest(self, closes: list[tuple[int, CloseCoefficient]]) -> None: ...


FINAL, KNOWN = "final", "known"


class FinalFirstAdmission(ContentReadyAdmission):
    def __init__(self, trainer: GroupLedgerTrainer, *, group_size: int, trainer_call: TrainerCall = direct_call,
                 final_forest: bool = False, known_reserve_slabs: int = 0,
                 events_waiting: Callable[[], bool] | None = None, **gates: Any) -> None:
        super().__init__(trainer, group_size=group_size, trainer_call=trainer_call, **gates)
        if known_reserve_slabs < 0:
            raise ValueError(f"known_reserve_slabs={known_reserve_slabs} is negative")
        if known_reserve_slabs and not self._gate.bounded:
            raise ValueError("known_reserve_slabs sets slabs aside within max_held_sources, so that budget must be set")
        self._ledger = trainer
        self._verdicts: Counter = Counter()
        self._forest = bool(final_forest)
        self._known_reserve_slabs = int(known_reserve_slabs)
        self._events_waiting = events_waiting
        self._paused = False  # set when this drain gave way to waiting events; cleared by the next drain

    # ---------------------------------------------------------------- classification
    def _is_final(self, group_id: int) -> bool:
        return self._verdicts[group_id] == self._group_size

    def _class_of(self, close: Close) -> str:
        return FINAL if self._is_final(close.group) else KNOWN

    def _events_pending(self) -> bool:
        """Whether trainer events are waiting now (remembered as a pause until the next drain)."""
        if self._events_waiting is not None and self._events_waiting():
            self._paused = True
            return True
        return False

    def _interrupted(self) -> bool:
        """True once this drain (or a later admission check) found trainer events waiting."""
        return self._events_pending() or self._paused

    # ---------------------------------------------------------------- events
    def bind_verdict(self, group_id: int, trajectory_id: int, reward: CloseCoefficient) -> None:
        self._verdicts[group_id] += 1
        if (group_id, trajectory_id) in self._waiting:
            self._ledger.record_rewards([(trajectory_id, reward)])
            self._to_close(group_id, trajectory_id, reward)
        else:
            super().bind_verdict(group_id, trajectory_id, reward)

    def _forest_ready(self) -> bool:
        return (self._forest and bool(self._closes) and not self._waiting
                and self._ledger.registered_groups_fully_bound()
                and all(self._class_of(c) == FINAL for c in self._closes))

    def _final_forest(self, closes: list[Close]) -> None:
        pairs = [(c.trajectory, c.coefficient) for c in closes]
        self._call("trajectory_backward", lambda: self._ledger.close_final_forest(pairs),
                   trajectory_count=len(pairs), trajectory_ids=[t for t, _ in pairs],
                   group_ids=sorted({c.group for c in closes}), job_class="final_forest")
        for c in closes:
            self._mark_bound(c.group)

    def drain_ready_closes(self) -> None:
        self._paused = False
        if self._forest_ready():
            backlog, self._closes = self._closes, []
            self._final_forest(backlog)
            return
        final = [c for c in self._closes if self._class_of(c) == FINAL]
        known = [c for c in self._closes if self._class_of(c) == KNOWN]
        if final:
            left = self._drain_final(final)
            if left or (known and self._interrupted()):
                self._closes = left + known
                return
        if self._known_reserve_slabs:
            self._closes = self._drain_known_reserved(known)
            return
        self._closes = self._drain(known, gated=True, job_class=KNOWN)

    def _drain_known_reserved(self, known: list[Close]) -> list[Close]:
        """With ``known_reserve_slabs``: known closes run outside the held-source budget (a known close
        holds no source that waits for a reward, so it never queues behind content work), at most the
        reserve per drain -- fewer when the trainer reports fewer free known slabs."""
        cap_fn = getattr(self._ledger, "known_slab_capacity", None)
        cap = cap_fn() if cap_fn is not None else None
        n = self._known_reserve_slabs if cap is None else min(self._known_reserve_slabs, max(0, int(cap)))
        if n == 0:
            return known
        return self._drain(known[:n], gated=False, job_class=KNOWN) + known[n:]

    def _drain_final(self, closes: list[Close]) -> list[Close]:
        """Final closes ignore the budget but give way to waiting events between packs."""
        rest = list(closes)
        size = self._pack_size(len(rest))
        while rest:
            rest = self._drain(rest[:size], gated=False, job_class=FINAL) + rest[size:]
            if rest and self._interrupted():
                break
        return rest

    def flush_prepares(self, *, force: bool = False) -> None:
        if self._paused and not force:
            return
        super().flush_prepares(force=force)

    def _may_admit(self, incoming: int, *, memory: bool = True) -> bool:
        if memory and self._interrupted():
            return False
        return super()._may_admit(incoming, memory=memory)

    def _launch_prepare(self, trajectories: list[int], groups: list[int], **labels: Any) -> None:
        super()._launch_prepare(trajectories, groups, job_class="content", **labels)
