"""GRPO admission: final work first, then known closes, then content (C43, GRPO).

A verdict for a completion still waiting to be prepared records the reward in
the trainer's ledger and turns the completion into a close -- *final* once
every verdict of its group has landed (its advantage is then known), *known*
otherwise. ``drain_ready_closes`` runs final closes at once and ungated, then
known closes under the residency budget; with ``final_forest`` a backlog that
is entirely final after the step's last verdict runs as one forest call.
Behaviour follows reference src/thundersync/grpo/admission.py:77-261.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Protocol

from thundersync_b200.scheduling.admission import CloseCoefficient, ContentReadyAdmission, EarlyTrainer, TrainerCall, direct_call

__all__ = ["GroupLedgerTrainer", "FinalFirstAdmission"]


class GroupLedgerTrainer(EarlyTrainer, Protocol):
    def record_rewards(self, binds: list[tuple[int, CloseCoefficient]]) -> None: ...
    def registered_groups_fully_bound(self) -> bool: ...
    def close_final_forest(self, closes: list[tuple[int, CloseCoefficient]]) -> None: ...


class FinalFirstAdmission(ContentReadyAdmission):
    def __init__(self, trainer: GroupLedgerTrainer, *, group_size: int, trainer_call: TrainerCall = direct_call,
                 final_forest: bool = False, known_reserve_slabs: int = 0,
                 events_waiting: Callable[[], bool] | None = None, **gates) -> None:
        super().__init__(trainer, group_size=group_size, trainer_call=trainer_call, **gates)
        if known_reserve_slabs < 0:
            raise ValueError("known_reserve_slabs must not be negative")
        if known_reserve_slabs and self._max_held_sources is None:
            raise ValueError("known_reserve_slabs reserves slabs beside the held-source budget, which is unset")
        self._ledger = trainer
        self._verdicts: dict[int, int] = {}
        self._final_forest = bool(final_forest)
        self._known_reserve_slabs = int(known_reserve_slabs)
        self._events_waiting = events_waiting
        self._yielded = False

    def _group_final(self, group_id: int) -> bool:
        return self._verdicts.get(group_id, 0) == self._group_size

    def _should_yield(self) -> bool:
        if self._events_waiting is not None and self._events_waiting():
            self._yielded = True
            return True
        return False

    def bind_verdict(self, group_id: int, trajectory_id: int, reward: CloseCoefficient) -> None:
        self._verdicts[group_id] = self._verdicts.get(group_id, 0) + 1
        if (group_id, trajectory_id) not in self._pending:
            super().bind_verdict(group_id, trajectory_id, reward)
            return
        self._ledger.record_rewards([(trajectory_id, reward)])
        self._defer_to_ready_close(group_id, trajectory_id, reward)

    def _final_forest_ready(self) -> bool:
        return (self._final_forest and bool(self._ready_close_queue) and not self._pending
                and self._ledger.registered_groups_fully_bound()
                and all(self._group_final(g) for g, _, _ in self._ready_close_queue))

    def _run_final_forest(self, backlog: list[tuple[int, int, CloseCoefficient]]) -> None:
        closes = [(t, r) for _, t, r in backlog]
        self._call("trajectory_backward", lambda: self._ledger.close_final_forest(closes),
                   trajectory_count=len(closes), trajectory_ids=[t for t, _ in closes],
                   group_ids=sorted({g for g, _, _ in backlog}), job_class="final_forest")
        for g, _, _ in backlog:
            self._record_bound(g)

    def drain_ready_closes(self) -> None:
        self._yielded = False
        if self._final_forest_ready():
            backlog, self._ready_close_queue = self._ready_close_queue, []
            self._run_final_forest(backlog)
            return
        final = [x for x in self._ready_close_queue if self._group_final(x[0])]
        if final:
            self._ready_close_queue = [x for x in self._ready_close_queue if not self._group_final(x[0])]
            rest = self._drain_yielding(final, job_class="final")
            if rest:
                self._ready_close_queue = rest + self._ready_close_queue
                return
            if self._ready_close_queue and self._should_yield():
                return
        self._drain_closes(self._ready_close_queue, gated=True, job_class="known")

    def _drain_yielding(self, queue, **labels):
        size = self._max_prepare_pack or max(1, len(queue))
        queue = list(queue)
        while queue:
            chunk, queue = queue[:size], queue[size:]
            self._drain_closes(chunk, gated=False, **labels)
            if queue and self._should_yield():
                return queue
        return []

    def flush_prepares(self, *, force: bool = False) -> None:
        if self._yielded and not force:
            return
        super().flush_prepares(force=force)

    def _admission_open(self, incoming: int, *, gate_memory: bool = True) -> bool:
        if gate_memory and (self._yielded or self._should_yield()):
            return False
        return super()._admission_open(incoming, gate_memory=gate_memory)

    def _prepare_pack(self, pack, group_ids, **labels) -> None:
        super()._prepare_pack(pack, group_ids, job_class="content", **labels)
