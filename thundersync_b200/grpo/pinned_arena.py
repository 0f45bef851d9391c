"""Bounded, reusable page-locked host slabs for offloaded sources and statistics (C31).

A rank that keeps GRPO sources or statistics on the host needs page-locked
memory for asynchronous device↔host copies, but pinning is slow, bounded by
the host, and shared by every rank on it. This module holds:

* ``host_pinned_budget`` — this rank's share of ``MemAvailable``:
  ``available · host_fraction / host_ranks − reserved`` (``host_ranks`` is
  torchrun's ``LOCAL_WORLD_SIZE``);
* ``PinnedSourceArena`` — slabs sized ``bytes + bytes/32`` rounded to the
  registration piece; ``acquire`` hands out the smallest free slab that
  fits, registers a new one while the byte budget and slab cap allow
  (replacing free slabs that are too small, largest first, when only that
  fits the budget), else waits for a ``release``; a wait that cannot end
  raises rather than hangs;
* ``PinnedStatisticPool`` — reusable (unit, reward) statistic homes for
  open groups, in a fixed per-parameter layout (512-byte aligned offsets).

Slabs come from this package's native allocator (``pinned_slab_alloc``): one
2 MiB-aligned host allocation registered with ``cudaHostRegister`` in pieces
of at most 4096 pages, all or nothing, under the device current when the
arena was built (reference: src/thundersync/grpo/pinned_arena.py:44-898; the
piece size, the slab headroom and the budget formula are kept because the
host-memory behaviour they encode is the point).
"""

from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

__all__ = [
    "PinnedSlab",
    "PinnedSourceArena",
    "PinnedStatisticPool",
    "StatisticSlot",
    "default_piece_bytes",
    "host_pinned_budget",
    "host_ranks_from_env",
    "read_mem_available_bytes",
    "registration_device",
    "tensor_offsets",
]

PIN_PIECE_PAGES = 4096
TENSOR_ALIGN_BYTES = 512
SLAB_HEADROOM_DIVISOR = 32
_WAIT_POLL_S = 0.05
DEFAULT_WAIT_TIMEOUT_S = 1800.0


def _round_up(v: int, m: int) -> int:
    return -(-v // m) * m


def _gib(v: float) -> float:
    return round(v / (1 << 30), 3)


def default_piece_bytes() -> int:
    return PIN_PIECE_PAGES * os.sysconf("SC_PAGE_SIZE")


def tensor_offsets(sizes: list[int]) -> tuple[list[int], int]:
    """512-byte aligned offset of each packed tensor and the packed total."""
    offs, cur = [], 0
    for s in sizes:
        cur = _round_up(cur, TENSOR_ALIGN_BYTES)
        offs.append(cur)
        cur += s
    return offs, cur


def registration_device() -> int | None:
    """The calling thread's CUDA device once CUDA is initialised, else None (no registration)."""
    if not torch.cuda.is_available() or not torch.cuda.is_initialized():
        return None
    return torch.cuda.current_device()


def read_mem_available_bytes(path: str = "/proc/meminfo") -> int:
    with open(path, encoding="utf-8") as fh:
        for line in fh:
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    raise RuntimeError(f"{path} does not report MemAvailable")


def host_ranks_from_env() -> int:
    value = os.environ.get("LOCAL_WORLD_SIZE", "1")
    n = int(value)
    if n < 1:
        raise ValueError(f"LOCAL_WORLD_SIZE must be positive, got {value}")
    return n


def host_pinned_budget(*, host_ranks: int, host_fraction: float, reserved_bytes: int,
                       available_bytes: int | None = None) -> tuple[int, dict[str, Any]]:
    """(budget bytes, evidence) for this rank's pinned sources."""
    if host_ranks < 1:
        raise ValueError("host_ranks must be positive")
    if not 0.0 < host_fraction <= 1.0:
        raise ValueError("host_fraction must be in (0, 1]")
    if reserved_bytes < 0:
        raise ValueError("reserved_bytes must not be negative")
    avail = read_mem_available_bytes() if available_bytes is None else available_bytes
    share = int(avail * host_fraction) // host_ranks
    budget = max(0, share - reserved_bytes)
    return budget, {"mem_available_bytes": avail, "host_fraction": host_fraction, "host_ranks": host_ranks,
                    "rank_share_bytes": share, "reserved_bytes": reserved_bytes, "budget_bytes": budget}


def _alloc(capacity: int, piece: int, device: int | None) -> tuple[torch.Tensor, int]:
    """A host slab of ``capacity`` bytes, page-locked when ``device`` is set."""
    from thundersync_b200.ops._ext import native

    ext = native()
    buf, pieces = ext.pinned_slab_alloc(int(capacity), int(piece), -1 if device is None else int(device))
    return buf, int(pieces)


@dataclass
class PinnedSlab:
    index: int
    capacity: int
    buffer: torch.Tensor
    pieces: int = 0
    owner: Any = None
    copy_event: Any = None


class PinnedSourceArena:
    """Page-locked slabs, one per unfolded source, under a byte budget and an optional slab cap."""

    def __init__(self, *, budget_bytes: int, max_slabs: int | None = None, piece_bytes: int | None = None,
                 wait_timeout_s: float = DEFAULT_WAIT_TIMEOUT_S, evidence: dict[str, Any] | None = None,
                 statistics: "PinnedStatisticPool | None" = None) -> None:
        page = os.sysconf("SC_PAGE_SIZE")
        piece = default_piece_bytes() if piece_bytes is None else piece_bytes
        if piece < page or piece % page:
            raise ValueError("piece_bytes must be a positive multiple of the page size")
        if piece > default_piece_bytes():
            raise ValueError(f"piece_bytes above {PIN_PIECE_PAGES} pages needs a costly-order kernel allocation per pin")
        if budget_bytes < 1:
            raise ValueError("budget_bytes must be positive")
        if max_slabs is not None and max_slabs < 1:
            raise ValueError("max_slabs must be positive when set")
        if wait_timeout_s <= 0.0:
            raise ValueError("wait_timeout_s must be positive")
        self._piece = piece
        self._budget = budget_bytes
        self._max_slabs = max_slabs
        self._timeout = wait_timeout_s
        self._evidence = dict(evidence or {})
        self._cv = threading.Condition()
        self._slabs: list[PinnedSlab] = []
        self._registered = 0
        self._pending = 0
        self._next = 0
        self._closed = False
        self._stats = {"acquires": 0, "waits": 0, "wait_s": 0.0, "max_wait_s": 0.0, "peak_busy_slabs": 0,
                       "peak_registered_bytes": 0, "register_s": 0.0, "registered_pieces": 0, "replaced_slabs": 0}
        self._busy = 0
        self.statistics = statistics
        self._device = registration_device()

    @classmethod
    def for_host(cls, source_bytes: int, *, host_ranks: int, host_fraction: float, reserved_bytes: int,
                 min_slabs: int, max_slabs: int | None, available_bytes: int | None = None,
                 piece_bytes: int | None = None, statistics: "PinnedStatisticPool | None" = None):
        """Size the arena from the host's MemAvailable; raises below ``min_slabs``."""
        if source_bytes < 1:
            raise ValueError("source_bytes must be positive")
        if min_slabs < 1:
            raise ValueError("min_slabs must be positive")
        budget, ev = host_pinned_budget(host_ranks=host_ranks, host_fraction=host_fraction,
                                        reserved_bytes=reserved_bytes, available_bytes=available_bytes)
        piece = default_piece_bytes() if piece_bytes is None else piece_bytes
        slab = cls.slab_capacity(source_bytes, piece)
        fits = budget // slab
        if fits < min_slabs:
            raise RuntimeError(
                f"pinned sources: this rank's host budget holds {fits} source slab(s), the configuration needs "
                f"{min_slabs}. MemAvailable {_gib(ev['mem_available_bytes'])} GiB x {host_fraction} / {host_ranks} "
                f"trainer rank(s) on this host = {_gib(ev['rank_share_bytes'])} GiB, minus {_gib(reserved_bytes)} GiB "
                f"of group statistics = {_gib(budget)} GiB; one slab is {_gib(slab)} GiB. Free host memory, run fewer "
                "ranks on this host, or lower max_held_sources / prepare_pack_max.")
        n = fits if max_slabs is None else min(fits, max_slabs)
        ev.update({"source_bytes": source_bytes, "slab_bytes": slab, "min_slabs": min_slabs,
                   "max_slabs_requested": max_slabs, "slabs_fit": fits})
        return cls(budget_bytes=budget, max_slabs=n, piece_bytes=piece, evidence=ev, statistics=statistics)

    @staticmethod
    def slab_capacity(nbytes: int, piece_bytes: int | None = None) -> int:
        piece = default_piece_bytes() if piece_bytes is None else piece_bytes
        return _round_up(max(1, nbytes + nbytes // SLAB_HEADROOM_DIVISOR), piece)

    @property
    def piece_bytes(self) -> int:
        return self._piece

    @property
    def slab_limit(self) -> int | None:
        with self._cv:
            return self._max_slabs

    # ------------------------------------------------------------------ locked helpers
    def _free_fit(self, nbytes: int) -> PinnedSlab | None:
        fit = [s for s in self._slabs if s.owner is None and s.capacity >= nbytes]
        return min(fit, key=lambda s: s.capacity) if fit else None

    def _victims(self, capacity: int) -> list[PinnedSlab] | None:
        victims, reg, count = [], self._registered, len(self._slabs) + self._pending
        free = sorted((s for s in self._slabs if s.owner is None), key=lambda s: s.capacity, reverse=True)
        while not ((self._max_slabs is None or count < self._max_slabs) and reg + capacity <= self._budget):
            if not free:
                return None
            v = free.pop(0)
            victims.append(v)
            reg -= v.capacity
            count -= 1
        return victims

    def _reserve(self, capacity: int) -> list[PinnedSlab] | None:
        victims = self._victims(capacity)
        if victims is None:
            return None
        for v in victims:
            self._slabs.remove(v)
            self._registered -= v.capacity
        self._registered += capacity
        self._pending += 1
        self._stats["peak_registered_bytes"] = max(self._stats["peak_registered_bytes"], self._registered)
        return victims

    def _progress(self, nbytes: int, capacity: int) -> bool:
        return self._free_fit(nbytes) is not None or bool(self._pending) or self._victims(capacity) is not None

    def _hand_out(self, slab: PinnedSlab, owner: Any, started: float, waited: bool) -> PinnedSlab:
        slab.owner = owner
        slab.copy_event = None
        self._stats["acquires"] += 1
        self._busy += 1
        self._stats["peak_busy_slabs"] = max(self._stats["peak_busy_slabs"], self._busy)
        if waited:
            dt = time.perf_counter() - started
            self._stats["waits"] += 1
            self._stats["wait_s"] += dt
            self._stats["max_wait_s"] = max(self._stats["max_wait_s"], dt)
        return slab

    def _register(self, capacity: int, owner: Any, victims: list[PinnedSlab], started: float, waited: bool):
        t0 = time.perf_counter()
        try:
            for v in victims:
                v.buffer = None  # the native deleter unregisters and frees
            buf, pieces = _alloc(capacity, self._piece, self._device)
        except BaseException:
            with self._cv:
                self._registered -= capacity
                self._pending -= 1
                self._cv.notify_all()
            raise
        with self._cv:
            self._pending -= 1
            slab = PinnedSlab(self._next, capacity, buf, pieces)
            self._next += 1
            self._slabs.append(slab)
            self._stats["register_s"] += time.perf_counter() - t0
            self._stats["registered_pieces"] += pieces
            self._stats["replaced_slabs"] += len(victims)
            return self._hand_out(slab, owner, started, waited)

    # ------------------------------------------------------------------ public
    def acquire(self, nbytes: int, *, owner: Any, release_possible: Callable[[], bool]) -> PinnedSlab:
        """A slab of at least ``nbytes``; waits for a release when none can be had.

        ``release_possible`` (called without the lock) reports whether a busy
        slab can still be released without this caller returning; when it
        cannot, the wait would never end and this raises.
        """
        if nbytes < 1:
            raise ValueError("a pinned slab request must be positive")
        cap = self.slab_capacity(nbytes, self._piece)
        started = time.perf_counter()
        waited = False
        while True:
            with self._cv:
                if self._closed:
                    raise RuntimeError("the pinned source arena is closed")
                slab = self._free_fit(nbytes)
                if slab is not None:
                    return self._hand_out(slab, owner, started, waited)
                plan = self._reserve(cap)
                if plan is None:
                    if self._busy == 0 and self._pending == 0:
                        raise RuntimeError(f"pinned sources: a {_gib(nbytes)} GiB source does not fit this rank's "
                                           f"{_gib(self._budget)} GiB pinned budget ({len(self._slabs)} slab(s), "
                                           f"{_gib(self._registered)} GiB registered)")
                    waited = True
                    self._cv.wait(timeout=_WAIT_POLL_S)
                    if self._progress(nbytes, cap):
                        continue
                    if time.perf_counter() - started > self._timeout:
                        raise RuntimeError(f"pinned sources: no slab was released within {self._timeout:.0f} s "
                                           f"({self._busy} of {len(self._slabs)} busy)")
            if plan is not None:
                return self._register(cap, owner, plan, started, waited)
            if release_possible():
                continue
            with self._cv:
                if self._progress(nbytes, cap):
                    continue
                busy = self._busy
            raise RuntimeError(
                "pinned sources: every busy slab holds a source that cannot fold until its reward is bound, and the "
                f"caller waiting for a slab is the one that binds rewards ({busy} busy of {self._max_slabs} slab(s), "
                f"{_gib(self._budget)} GiB budget). Raise the host budget or keep max_held_sources and "
                "prepare_pack_max at or below the arena's slab count.")

    def try_acquire(self, nbytes: int, *, owner: Any) -> PinnedSlab | None:
        if nbytes < 1:
            raise ValueError("a pinned slab request must be positive")
        cap = self.slab_capacity(nbytes, self._piece)
        started = time.perf_counter()
        with self._cv:
            if self._closed:
                raise RuntimeError("the pinned source arena is closed")
            slab = self._free_fit(nbytes)
            if slab is not None:
                return self._hand_out(slab, owner, started, False)
            plan = self._reserve(cap)
            if plan is None:
                return None
        return self._register(cap, owner, plan, started, False)

    def release(self, slab: PinnedSlab) -> None:
        """Return a slab once any copy still writing into it has completed."""
        if slab.copy_event is not None:
            slab.copy_event.synchronize()
        with self._cv:
            if self._closed:
                slab.owner = None
                return
            if slab.owner is None:
                raise RuntimeError("pinned slab released twice")
            slab.owner = None
            slab.copy_event = None
            self._busy -= 1
            self._cv.notify_all()

    def copy_into(self, slab: PinnedSlab, offset: int, value: torch.Tensor) -> torch.Tensor:
        """Enqueue ``value``'s device→host copy on the current stream; returns the typed slab view."""
        if value.device.type != "cuda":
            raise RuntimeError("pinned slab copies take CUDA sources")
        if not value.is_contiguous():
            raise RuntimeError("pinned slab copies take contiguous sources")
        nbytes = value.numel() * value.element_size()
        if offset < 0 or offset % TENSOR_ALIGN_BYTES or offset + nbytes > slab.capacity:
            raise RuntimeError("pinned slab copy is outside the slab")
        dst = slab.buffer[offset:offset + nbytes]
        if nbytes:
            dst.copy_(value.reshape(-1).view(torch.uint8), non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            slab.copy_event = ev
        return dst.view(value.dtype).view(value.shape)

    def extend_slab_limit(self, count: int) -> int:
        if count < 1:
            raise ValueError("the slab cap extension must be positive")
        with self._cv:
            if self._max_slabs is None:
                raise RuntimeError("the arena has no slab cap to extend: its byte budget alone bounds it")
            new = self._max_slabs + count
            fits = self._evidence.get("slabs_fit")
            if fits is not None and new > int(fits):
                raise RuntimeError(f"pinned sources: {new} slabs requested, this rank's host budget holds {fits} "
                                   f"({_gib(self._budget)} GiB); free host memory or lower known_reserve_slabs")
            self._max_slabs = new
            self._evidence["max_slabs_extended_by"] = int(self._evidence.get("max_slabs_extended_by", 0)) + count
            return new

    def close(self) -> None:
        with self._cv:
            if self._closed:
                return
            self._closed = True
            slabs, self._slabs = self._slabs, []
            self._registered = 0
            self._busy = 0
            self._cv.notify_all()
        for s in slabs:
            if s.copy_event is not None:
                s.copy_event.synchronize()
            s.buffer = None
        if self.statistics is not None:
            self.statistics.close()

    def report(self) -> dict[str, Any]:
        with self._cv:
            return {"piece_bytes": self._piece, "budget_bytes": self._budget, "max_slabs": self._max_slabs,
                    "slabs": len(self._slabs), "slab_capacities": [s.capacity for s in self._slabs],
                    "registered_bytes": self._registered, "busy_slabs": self._busy, **self._stats,
                    "host_budget": dict(self._evidence),
                    "statistics": None if self.statistics is None else self.statistics.report()}


@dataclass
class StatisticSlot:
    index: int
    unit: torch.Tensor
    reward: torch.Tensor
    owner: Any = None
    reload_event: Any = None
    pieces: int = 0


class PinnedStatisticPool:
    """Reusable page-locked (unit, reward) statistic homes, at most ``slots`` of them.

    A slot is built on its first acquire and kept until ``close``. ``acquire``
    returns None when every slot is owned (the group then allocates its
    statistics as usual); ``release`` takes the event of the last reload copy,
    which the next acquire of that slot waits for.
    """

    def __init__(self, element_counts: list[int], dtype: torch.dtype, *, slots: int,
                 piece_bytes: int | None = None) -> None:
        if slots < 1:
            raise ValueError("a statistic pool needs at least one slot")
        page = os.sysconf("SC_PAGE_SIZE")
        piece = default_piece_bytes() if piece_bytes is None else piece_bytes
        if piece < page or piece % page or piece > default_piece_bytes():
            raise ValueError(f"piece_bytes must be a page multiple of at most {PIN_PIECE_PAGES} pages")
        if any(c < 0 for c in element_counts):
            raise ValueError("element counts must not be negative")
        self.element_counts = [int(c) for c in element_counts]
        self.dtype = dtype
        es = torch.empty((), dtype=dtype).element_size()
        self._sizes = [c * es for c in self.element_counts]
        self._offsets, total = tensor_offsets(self._sizes)
        self._capacity = _round_up(max(1, total), piece)
        self._piece = piece
        self._max = slots
        self._lock = threading.Lock()
        self._slots: list[StatisticSlot] = []
        self._building = 0
        self._next = 0
        self._closed = False
        self._acquires = self._misses = self._busy = self._peak = 0
        self._build_s = 0.0
        self._device = registration_device()

    @property
    def slot_bytes(self) -> int:
        return 2 * self._capacity

    def acquire(self, owner: Any) -> StatisticSlot | None:
        with self._lock:
            if self._closed:
                raise RuntimeError("the statistic pool is closed")
            slot = next((s for s in self._slots if s.owner is None), None)
            if slot is None:
                if len(self._slots) + self._building >= self._max:
                    self._misses += 1
                    return None
                self._building += 1
            else:
                slot.owner = owner
                self._count()
        if slot is None:
            try:
                t0 = time.perf_counter()
                unit, pu = _alloc(self._capacity, self._piece, self._device)
                reward, pr = _alloc(self._capacity, self._piece, self._device)
            finally:
                with self._lock:
                    self._building -= 1
            with self._lock:
                slot = StatisticSlot(self._next, unit, reward, owner, None, pu + pr)
                self._next += 1
                self._build_s += time.perf_counter() - t0
                self._slots.append(slot)
                self._count()
        if slot.reload_event is not None:
            slot.reload_event.synchronize()
            slot.reload_event = None
        return slot

    def _count(self) -> None:
        self._acquires += 1
        self._busy += 1
        self._peak = max(self._peak, self._busy)

    def fits(self, index: int, value: torch.Tensor) -> bool:
        return 0 <= index < len(self.element_counts) and value.numel() == self.element_counts[index]

    def view(self, slot: StatisticSlot, index: int, shape: torch.Size, *, statistic: str) -> torch.Tensor:
        buf = {"unit": slot.unit, "reward": slot.reward}[statistic]
        a = self._offsets[index]
        return buf[a:a + self._sizes[index]].view(self.dtype).view(shape)

    def reload_reward(self, slot: StatisticSlot, index: int, shape: torch.Size, device: torch.device) -> torch.Tensor:
        """Enqueue parameter ``index``'s reward statistic host→device on the current stream."""
        out = torch.empty(shape, dtype=self.dtype, device=device)
        n = self._sizes[index]
        if n:
            a = self._offsets[index]
            out.view(-1).view(torch.uint8).copy_(slot.reward[a:a + n], non_blocking=True)
        return out

    def release(self, slot: StatisticSlot, *, reload_event: Any = None) -> None:
        with self._lock:
            if self._closed:
                slot.owner = None
                return
            if slot.owner is None:
                raise RuntimeError("statistic slot released twice")
            slot.owner = None
            slot.reload_event = reload_event
            self._busy -= 1

    def report(self) -> dict[str, Any]:
        with self._lock:
            return {"max_slots": self._max, "slots": len(self._slots), "slot_bytes": self.slot_bytes,
                    "registered_bytes": len(self._slots) * 2 * self._capacity, "busy_slots": self._busy,
                    "peak_busy_slots": self._peak, "acquires": self._acquires, "misses": self._misses,
                    "build_s": self._build_s, "dtype": str(self.dtype)}

    def close(self) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
            slots, self._slots = self._slots, []
            self._busy = 0
        for s in slots:
            if s.reload_event is not None:
                s.reload_event.synchronize()
            s.unit = s.reward = None
