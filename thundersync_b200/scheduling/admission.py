"""Content-ready admission: prepare at completion, bind at verdict (C43, generic).

``add_completion`` queues a content-ready trajectory; ``flush_prepares`` runs
queued completions as packed branch backwards (``max_prepare_pack`` bounds a
pack, ``max_held_sources`` bounds differentiated-but-unfolded sources using
the trainer's own count). ``bind_verdict`` attaches the reward (a lock-free
ledger update, not a backward). A verdict that lands before its completion
was prepared becomes a *ready close* (backward with the reward known) that
drains under the same budget. Group closes never block ingestion:
``close_ready_groups`` closes only groups whose reduction already finished;
``drain_group_closes`` closes the rest at the batch boundary. Behaviour
follows reference src/thundersync/scheduling/admission.py:65-363.
"""

from __future__ import annotations

from collections.abc import Callable
from typing import Any, Protocol

__all__ = ["CloseCoefficient", "TrainerCall", "EarlyTrainer", "ContentReadyAdmission", "direct_call"]

CloseCoefficient = float | None


class TrainerCall(Protocol):
    def __call__(self, kind: str, fn: Callable[[], Any], **labels: Any) -> Any: ...


def direct_call(kind: str, fn: Callable[[], Any], **labels: Any) -> Any:
    """The trivial ``trainer_call``: run the call now."""
    return fn()


class EarlyTrainer(Protocol):
    def prepare_trajectories(self, trajectory_ids: list[int]) -> None: ...
    def bind_rewards(self, binds: list[tuple[int, CloseCoefficient]]) -> None: ...
    def close_trajectories(self, closes: list[tuple[int, CloseCoefficient]]) -> None: ...
    def close_group(self, group_id: int) -> None: ...
    def group_reduction_complete(self, group_id: int) -> bool: ...


class ContentReadyAdmission:
    def __init__(self, trainer: EarlyTrainer, *, group_size: int, trainer_call: TrainerCall = direct_call,
                 max_prepare_pack: int | None = None, max_held_sources: int | None = None,
                 in_flight_sources: Callable[[], int] | None = None,
                 memory_pressure: Callable[[], bool] | None = None) -> None:
        if max_prepare_pack is not None and max_prepare_pack < 1:
            raise ValueError("max_prepare_pack must be positive when set")
        if max_held_sources is not None and max_held_sources < 1:
            raise ValueError("max_held_sources must be positive when set")
        if max_held_sources is not None and in_flight_sources is None:
            raise ValueError("max_held_sources needs in_flight_sources: the budget must release on fold completion")
        self._trainer = trainer
        self._group_size = group_size
        self._call = trainer_call
        self._max_prepare_pack = max_prepare_pack
        self._max_held_sources = max_held_sources
        self._in_flight = in_flight_sources
        self._pressure = memory_pressure
        self._pending: list[tuple[int, int]] = []  # (group, trajectory) awaiting prepare
        self._ready_close_queue: list[tuple[int, int, CloseCoefficient]] = []
        self._bound: dict[int, int] = {}
        self._pending_group_closes: list[int] = []

    # ---------------------------------------------------------------- helpers
    @property
    def _pending_prepares(self) -> list[int]:
        return [t for _, t in self._pending]

    def _admission_open(self, incoming: int, *, gate_memory: bool = True) -> bool:
        if gate_memory and self._pressure is not None and self._pressure():
            return False
        if self._max_held_sources is None:
            return True
        return self._in_flight() + incoming <= self._max_held_sources

    def _prepare_pack(self, pack: list[int], group_ids: list[int], **labels: str) -> None:
        self._call("trajectory_backward", lambda: self._trainer.prepare_trajectories(pack),
                   trajectory_count=len(pack), trajectory_ids=list(pack), group_ids=group_ids, **labels)

    def _record_bound(self, group_id: int) -> None:
        self._bound[group_id] = self._bound.get(group_id, 0) + 1
        if self._bound[group_id] == self._group_size:
            self._pending_group_closes.append(group_id)

    def _defer_to_ready_close(self, group_id: int, trajectory_id: int, reward: CloseCoefficient) -> None:
        self._pending.remove((group_id, trajectory_id))
        self._ready_close_queue.append((group_id, trajectory_id, reward))

    # ---------------------------------------------------------------- events
    def add_completion(self, group_id: int, trajectory_id: int) -> None:
        self._pending.append((group_id, trajectory_id))

    def flush_prepares(self, *, force: bool = False) -> None:
        if not self._pending:
            return
        todo, self._pending = self._pending, []
        size = self._max_prepare_pack or len(todo)
        for i in range(0, len(todo), size):
            chunk = todo[i : i + size]
            if not force and not self._admission_open(len(chunk)):
                self._pending = todo[i:]
                return
            self._prepare_pack([t for _, t in chunk], sorted({g for g, _ in chunk}))

    def bind_verdict(self, group_id: int, trajectory_id: int, reward: CloseCoefficient) -> None:
        if (group_id, trajectory_id) in self._pending:
            if self._max_held_sources is None:
                self.flush_prepares()
            else:
                self._defer_to_ready_close(group_id, trajectory_id, reward)
                return
        self._call("reward_bind", lambda: self._trainer.bind_rewards([(trajectory_id, reward)]),
                   trajectory_id=trajectory_id, group_id=group_id)
        self._record_bound(group_id)

    def drain_ready_closes(self) -> None:
        self._drain_closes(self._ready_close_queue, gated=True)

    def _drain_closes(self, queue: list[tuple[int, int, CloseCoefficient]], *, gated: bool, **labels: str) -> None:
        size = self._max_prepare_pack or max(1, len(queue))
        while queue:
            chunk = queue[:size]
            if gated and not self._admission_open(len(chunk), gate_memory=False):
                return
            del queue[: len(chunk)]
            closes = [(t, r) for _, t, r in chunk]
            self._call("trajectory_backward", lambda c=closes: self._trainer.close_trajectories(c),
                       trajectory_count=len(closes), trajectory_ids=[t for t, _ in closes],
                       group_ids=sorted({g for g, _, _ in chunk}), **labels)
            for g, _, _ in chunk:
                self._record_bound(g)

    @property
    def ready_close_backlog(self) -> int:
        return len(self._ready_close_queue)

    @property
    def deferred_work_reason(self) -> str | None:
        if self._ready_close_queue:
            return "ready_close"
        if self._pending:
            return "prepare"
        if self._pending_group_closes:
            return "group_close"
        return None

    def close_ready_groups(self) -> None:
        keep = []
        for gid in self._pending_group_closes:
            if self._trainer.group_reduction_complete(gid):
                self._call("group_close", lambda g=gid: self._trainer.close_group(g), group_id=gid)
            else:
                keep.append(gid)
        self._pending_group_closes = keep

    def drain_group_closes(self) -> None:
        if self._pending:
            raise RuntimeError("content-ready admission drained with unflushed preparations")
        if self._ready_close_queue:
            raise RuntimeError("content-ready admission drained with queued ready closes")
        for gid in self._pending_group_closes:
            self._call("group_close", lambda g=gid: self._trainer.close_group(g), group_id=gid)
        self._pending_group_closes = []
