"""Preallocated device homes for open groups' GRPO statistic pairs (C32).

One slot holds a group's two flat fp32 statistics (Σ∇S and Σr∇S — or the
binary P/N pair) in the parameter-arena layout, so a group's statistics are
two views, and the fold/combine kernels run on them unchanged. Every slot is
allocated at construction; ``acquire`` never waits (None when every slot is
owned — the group then allocates its pair on the statistic device as
usual); ``release`` takes an event after the group's last read, which the
next ``acquire`` of that slot waits for (reference:
src/thundersync/grpo/device_statistics.py:41-247).

``device_statistic_slots`` sizes the pool from what the device must hold
beside it: parameters, one gradient, this rank's optimizer state, the
resident unfolded sources and a reserve.
"""

from __future__ import annotations

import threading
from typing import Any

import torch

from thundersync_b200.grpo.pinned_arena import StatisticSlot

__all__ = ["DeviceStatisticPool", "device_statistic_slots"]


class DeviceStatisticPool:
    def __init__(self, numel: int, dtype: torch.dtype = torch.float32, *, slots: int,
                 device: torch.device | str) -> None:
        if isinstance(slots, bool) or not isinstance(slots, int) or slots < 1:
            raise ValueError("a device statistic pool needs at least one slot")
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("device statistic homes live on a CUDA device")
        if dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        if numel < 0:
            raise ValueError("numel must not be negative")
        self.numel = int(numel)
        self.dtype = dtype
        self.device = dev
        self._lock = threading.Lock()
        self._closed = False
        self._acquires = self._misses = self._busy = self._peak = 0
        self._slots = [StatisticSlot(i, torch.empty(self.numel, dtype=dtype, device=dev),
                                     torch.empty(self.numel, dtype=dtype, device=dev)) for i in range(slots)]

    @property
    def slot_bytes(self) -> int:
        return 2 * self.numel * torch.empty((), dtype=self.dtype).element_size()

    @property
    def slots(self) -> int:
        return len(self._slots)

    def acquire(self, owner: Any) -> StatisticSlot | None:
        """A free slot (both homes zeroed on the current stream), or None."""
        with self._lock:
            if self._closed:
                raise RuntimeError("the device statistic pool is closed")
            slot = next((s for s in self._slots if s.owner is None), None)
            if slot is None:
                self._misses += 1
                return None
            slot.owner = owner
            self._acquires += 1
            self._busy += 1
            self._peak = max(self._peak, self._busy)
        if slot.reload_event is not None:
            torch.cuda.current_stream(self.device).wait_event(slot.reload_event)
            slot.reload_event = None
        slot.unit.zero_()
        slot.reward.zero_()
        return slot

    def owns(self, t: torch.Tensor | None) -> StatisticSlot | None:
        if t is None:
            return None
        for s in self._slots:
            if s.owner is not None and (s.unit.data_ptr() == t.data_ptr() or s.reward.data_ptr() == t.data_ptr()):
                return s
        return None

    def release(self, slot: StatisticSlot, *, reload_event: Any = None) -> None:
        with self._lock:
            if self._closed:
                slot.owner = None
                return
            if slot.owner is None:
                raise RuntimeError("statistic slot released twice")
            slot.owner = None
            if reload_event is None and torch.cuda.is_available():
                reload_event = torch.cuda.Event()
                reload_event.record(torch.cuda.current_stream(self.device))
            slot.reload_event = reload_event
            self._busy -= 1

    def report(self) -> dict[str, Any]:
        with self._lock:
            return {"slots": len(self._slots), "slot_bytes": self.slot_bytes, "busy_slots": self._busy,
                    "peak_busy_slots": self._peak, "acquires": self._acquires, "misses": self._misses,
                    "dtype": str(self.dtype), "device": str(self.device)}

    def close(self) -> None:
        with self._lock:
            self._closed = True
            slots, self._slots = self._slots, []
            self._busy = 0
        for s in slots:
            if s.reload_event is not None:
                s.reload_event.synchronize()


def device_statistic_slots(*, device_total_bytes: int, parameter_bytes: int, gradient_bytes: int,
                           optimizer_state_bytes: int, source_bytes: int, device_held_sources: int,
                           statistic_pair_bytes: int, reserve_bytes: int, open_groups: int) -> int:
    """``min(open_groups, ⌊(device − params − grad − optimizer − held sources − reserve) / pair⌋)``."""
    vals = {"device_total_bytes": device_total_bytes, "parameter_bytes": parameter_bytes,
            "gradient_bytes": gradient_bytes, "optimizer_state_bytes": optimizer_state_bytes,
            "source_bytes": source_bytes, "device_held_sources": device_held_sources,
            "reserve_bytes": reserve_bytes, "open_groups": open_groups}
    for k, v in vals.items():
        if isinstance(v, bool) or not isinstance(v, int) or v < 0:
            raise ValueError(f"{k} must be a non-negative integer")
    if isinstance(statistic_pair_bytes, bool) or not isinstance(statistic_pair_bytes, int) or statistic_pair_bytes < 1:
        raise ValueError("statistic_pair_bytes must be a positive integer")
    room = (device_total_bytes - parameter_bytes - gradient_bytes - optimizer_state_bytes
            - device_held_sources * source_bytes - reserve_bytes)
    return 0 if room <= 0 else min(open_groups, room // statistic_pair_bytes)
