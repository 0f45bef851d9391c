"""Group-granular micro-batch packing for final (batch-ready) GRPO work (C34).

Groups in canonical group-id order, each kept whole, are packed greedily under
a logical-token budget; a group larger than the budget is its own micro-batch,
or with ``split_oversized_groups`` is cut into consecutive trajectory runs that
each fit (a single trajectory over budget stays alone). Torch-free; items need
``group_id``, ``traj_id`` and ``n_tokens``. Same rule as reference
src/thundersync/grpo/packing.py:43-85.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Protocol, TypeVar

__all__ = ["Packable", "pack_groups"]


class Packable(Protocol):
    @property
    def group_id(self) -> int: ...

    @property
    def traj_id(self) -> int: ...

    @property
    def n_tokens(self) -> int: ...


T = TypeVar("T", bound=Packable)


def pack_groups(trajectories: Sequence[T], *, max_tokens_per_microbatch: int,
                split_oversized_groups: bool = False) -> list[list[T]]:
    if max_tokens_per_microbatch < 1:
        raise ValueError("GRPO microbatch token budget must be positive")
    groups: dict[int, list[T]] = {}
    for t in trajectories:
        groups.setdefault(t.group_id, []).append(t)
    batches: list[list[T]] = []
    cur: list[T] = []
    cur_tokens = 0

    def flush() -> None:
        nonlocal cur, cur_tokens
        if cur:
            batches.append(cur)
        cur, cur_tokens = [], 0

    for gid in sorted(groups):
        members = sorted(groups[gid], key=lambda x: x.traj_id)
        size = sum(m.n_tokens for m in members)
        if split_oversized_groups and size > max_tokens_per_microbatch:
            flush()
            run: list[T] = []
            run_tokens = 0
            for m in members:
                if run and run_tokens + m.n_tokens > max_tokens_per_microbatch:
                    batches.append(run)
                    run, run_tokens = [], 0
                run.append(m)
                run_tokens += m.n_tokens
            batches.append(run)
            continue
        if cur and cur_tokens + size > max_tokens_per_microbatch:
            flush()
        cur.extend(members)
        cur_tokens += size
    flush()
    return batches
