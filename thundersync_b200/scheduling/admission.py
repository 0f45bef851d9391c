"""Content-ready admission: prepare at completion, bind at verdict (C43, generic).

Behaviour (matching reference src/thundersync/scheduling/admission.py:65-363):
a completed trajectory is queued; ``flush_prepares`` turns queued
completions into packed branch backwards, ``max_prepare_pack`` per pack and,
with ``max_held_sources``, never more differentiated-but-unfolded sources
than that budget (the trainer's own count, read through
``in_flight_sources``). ``bind_verdict`` attaches the reward, which is a
ledger update rather than a backward. A verdict that arrives while its
completion still waits (and a budget is set) makes the trajectory a *ready
close*: one backward with the reward known, drained under the same budget.
A group whose every trajectory is bound becomes closable; ``close_ready_groups``
closes only those whose reduction has already finished (ingestion never
waits on a group close) and ``drain_group_closes`` closes the rest at the
batch boundary.

Structure: completions wait in an insertion-ordered dict, ready closes in a
list of :class:`Close` records, the budget lives in a :class:`ResidencyGate`,
and every trainer call goes through one ``trainer_call`` hook with labels
(job kind, ids) so a caller can time or trace it. Subclasses extend the
policy through the ``_may_admit`` / ``_launch_prepare`` / ``_launch_closes`` /
``_drain`` / ``_mark_bound`` hooks.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Callable
from dataclasses import dataclass
from typing import Any, Protocol

__all__ = ["Close", "CloseCoefficient", "ContentReadyAdmission", "EarlyTrainer", "ResidencyGate", "TrainerCall",
           "direct_call"]

# What a close carries without the scheduler reading it: the reward for GRPO,
# None for on-policy distillation (whose supervision arrived per turn).
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


@dataclass(frozen=True)
class Close:
    """A trajectory whose reward is known and whose backward has not run."""

    group: int
    trajectory: int
    coefficient: CloseCoefficient


class ResidencyGate:
    """How many sources may be in flight, and whether device memory is under pressure."""

    def __init__(self, max_held_sources: int | None, in_flight_sources: Callable[[], int] | None,
                 memory_pressure: Callable[[], bool] | None) -> None:
        if max_held_sources is not None and max_held_sources < 1:
            raise ValueError(f"max_held_sources={max_held_sources}: give a positive budget or None")
        if max_held_sources is not None and in_flight_sources is None:
            raise ValueError("a max_held_sources budget needs in_flight_sources (the trainer's own count, "
                             "which drops as folds complete)")
        self.limit = max_held_sources
        self._count = in_flight_sources
        self._pressure = memory_pressure

    @property
    def bounded(self) -> bool:
        return self.limit is not None

    def admits(self, incoming: int, *, memory: bool = True) -> bool:
        if memory and self._pressure is not None and self._pressure():
            return False
        return self.limit is None or self._count() + incoming <= self.limit


class ContentReadyAdmission:
    """Early-training admission for one logical batch."""

    def __init__(self, trainer: EarlyTrainer, *, group_size: int, trainer_call: TrainerCall = direct_call,
                 max_prepare_pack: int | None = None, max_held_sources: int | None = None,
                 in_flight_sources: Callable[[], int] | None = None,
                 memory_pressure: Callable[[], bool] | None = None) -> None:
        if max_prepare_pack is not None and max_prepare_pack < 1:
            raise ValueError(f"max_prepare_pack={max_prepare_pack}: give a positive pack size or None")
        self._trainer = trainer
        self._group_size = int(group_size)
        self._call = trainer_call
        self._pack = max_prepare_pack
        self._gate = ResidencyGate(max_held_sources, in_flight_sources, memory_pressure)
        self._waiting: dict[tuple[int, int], None] = {}  # (group, trajectory) completions, arrival order
        self._closes: list[Close] = []
        self._bound: Counter = Counter()
        self._closable: list[int] = []

    # ---------------------------------------------------------------- hooks
    def _may_admit(self, incoming: int, *, memory: bool = True) -> bool:
        return self._gate.admits(incoming, memory=memory)

    def _pack_size(self, n: int) -> int:
        return self._pack or max(1, n)

    def _launch_prepare(self, trajectories: list[int], groups: list[int], **labels: Any) -> None:
        self._call("trajectory_backward", lambda: self._trainer.prepare_trajectories(trajectories),
                   trajectory_count=len(trajectories), trajectory_ids=list(trajectories), group_ids=groups,
                   **labels)

    def _launch_closes(self, closes: list[Close], **labels: Any) -> None:
        pairs = [(c.trajectory, c.coefficient) for c in closes]
        self._call("trajectory_backward", lambda: self._trainer.close_trajectories(pairs),
                   trajectory_count=len(pairs), trajectory_ids=[t for t, _ in pairs],
                   group_ids=sorted({c.group for c in closes}), **labels)
        for c in closes:
            self._mark_bound(c.group)

    def _mark_bound(self, group_id: int) -> None:
        self._bound[group_id] += 1
        if self._bound[group_id] == self._group_size:
            self._closable.append(group_id)

    def _drain(self, closes: list[Close], *, gated: bool, **labels: Any) -> list[Close]:
        """Run ``closes`` in packs; with ``gated`` stop at the first pack the budget refuses.
        Returns what was not run."""
        rest = list(closes)
        size = self._pack_size(len(rest))
        while rest:
            pack = rest[:size]
            if gated and not self._may_admit(len(pack), memory=False):
                break
            rest = rest[size:]
            self._launch_closes(pack, **labels)
        return rest

    def _to_close(self, group_id: int, trajectory_id: int, reward: CloseCoefficient) -> None:
        del self._waiting[(group_id, trajectory_id)]
        self._closes.append(Close(group_id, trajectory_id, reward))

    @property
    def _pending_prepares(self) -> list[int]:
        return [t for _, t in self._waiting]

    # ---------------------------------------------------------------- events
    def add_completion(self, group_id: int, trajectory_id: int) -> None:
        self._waiting[(group_id, trajectory_id)] = None

    def flush_prepares(self, *, force: bool = False) -> None:
        """Prepare waiting completions in packs while the budget admits them (``force`` ignores it)."""
        queue = list(self._waiting)
        size = self._pack_size(len(queue))
        for start in range(0, len(queue), size):
            pack = queue[start:start + size]
            if not force and not self._may_admit(len(pack)):
                return
            for key in pack:
                del self._waiting[key]
            self._launch_prepare([t for _, t in pack], sorted({g for g, _ in pack}))

    def bind_verdict(self, group_id: int, trajectory_id: int, reward: CloseCoefficient) -> None:
        if (group_id, trajectory_id) in self._waiting:
            if self._gate.bounded:
                self._to_close(group_id, trajectory_id, reward)
                return
            self.flush_prepares()
        self._call("reward_bind", lambda: self._trainer.bind_rewards([(trajectory_id, reward)]),
                   trajectory_id=trajectory_id, group_id=group_id)
        self._mark_bound(group_id)

    def drain_ready_closes(self) -> None:
        self._closes = self._drain(self._closes, gated=True)

    @property
    def ready_close_backlog(self) -> int:
        return len(self._closes)

    @property
    def deferred_work_reason(self) -> str | None:
        """What still waits: ``ready_close``, ``prepare``, ``group_close`` or nothing."""
        for reason, queue in (("ready_close", self._closes), ("prepare", self._waiting),
                              ("group_close", self._closable)):
            if queue:
                return reason
        return None

    def _close_group(self, group_id: int) -> None:
        self._call("group_close", lambda: self._trainer.close_group(group_id), group_id=group_id)

    def close_ready_groups(self) -> None:
        later = []
        for gid in self._closable:
            if self._trainer.group_reduction_complete(gid):
                self._close_group(gid)
            else:
                later.append(gid)
        self._closable = later

    def drain_group_closes(self) -> None:
        if self._waiting or self._closes:
            what = "completions that were never prepared" if self._waiting else "ready closes that never ran"
            raise RuntimeError(f"batch boundary reached with {what}")
        for gid in self._closable:
            self._close_group(gid)
        self._closable = []
