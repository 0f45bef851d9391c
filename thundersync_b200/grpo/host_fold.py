"""Host-resident GRPO statistics: overlapped device->host folds and host->device combines (C30/C31).

When a group's statistics live in host memory (``source_offload_device="cpu"``)
a trajectory's fp32 gradient (its *source*, on the device) must be folded
into the host pair ``G1 += r·g, G2 += g`` and, at the group close, the pair
must come back as one combined vector ``a·G1 + b·G2``. Doing either as one
blocking multi-GB copy stalls the device queue and leaves the host's memory
bandwidth idle, so :class:`HostFoldPipeline` streams them through a ring of
page-locked windows (reference behaviour: src/thundersync/grpo/reward_linear.py
:1003-1048 windows, :4763 offload workers, :4908 reducer workers):

* ``fold``: for each window-sized slice of the source, a device->host copy on
  a dedicated copy stream, then a host task that waits for that copy and adds
  the slice into the statistics (split across ``reduction_workers`` threads).
  The caller's stream only waits for the copies before it reuses the source
  buffer; the host folds run behind it.
* ``combine_into``: for each slice, host threads write ``a·G1 + b·G2`` into a
  window, which is copied host->device and added into the device gradient.

Windows come from a :class:`~thundersync_b200.grpo.pinned_arena.PinnedSourceArena`
when one is given (so they count against the rank's pinned budget), else from
torch's pinned allocator. Host statistics can be file-backed (``spill_dir``:
memory-mapped files, for hosts whose RAM cannot hold every open group's pair)
and can be kept in the parameters' dtype (``dtype``).
"""

from __future__ import annotations

import os
import tempfile
import threading
from concurrent.futures import Future, ThreadPoolExecutor
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

import torch

__all__ = ["HostFoldPipeline", "host_statistic"]


def host_statistic(numel: int, dtype: torch.dtype, spill_dir: str | os.PathLike | None) -> torch.Tensor:
    """A zeroed host vector; memory-mapped from a fresh file under ``spill_dir`` when one is set."""
    if spill_dir is None:
        return torch.zeros(numel, dtype=dtype)
    Path(spill_dir).mkdir(parents=True, exist_ok=True)
    fd, path = tempfile.mkstemp(prefix="ts-statistic-", suffix=".bin", dir=spill_dir)
    os.close(fd)
    t = torch.from_file(path, shared=True, size=numel, dtype=dtype)  # zero-filled sparse file
    os.unlink(path)  # the mapping keeps the pages; nothing is left on disk after the tensor dies
    return t


@dataclass
class _Window:
    buf: torch.Tensor  # page-locked bytes
    slab: Any = None  # arena slab backing ``buf`` (returned at close)
    copied: Any = None  # CUDA event: the copy into/out of this window finished
    pending: list[Future] = field(default_factory=list)  # host work still reading/writing this window


class HostFoldPipeline:
    """Streams fp32 device sources into host statistics and combined statistics back to the device."""

    def __init__(self, device: torch.device, *, window_bytes: int = 256 << 20, windows: int = 2,
                 offload_workers: int = 2, reduction_workers: int = 2, arena: Any = None) -> None:
        if window_bytes < 4096 or windows < 1 or offload_workers < 1 or reduction_workers < 1:
            raise ValueError("host fold pipeline: window_bytes >= 4096 and positive window/worker counts required")
        if device.type != "cuda":
            raise ValueError("the host fold pipeline streams from a CUDA device")
        self.device = device
        self.window_elems = window_bytes // 4
        self._ring: list[_Window] = []
        for i in range(windows):
            if arena is not None:
                slab = arena.acquire(window_bytes, owner=("host-fold-window", i), release_possible=lambda: False)
                self._ring.append(_Window(slab.buffer[:window_bytes], slab))
            else:
                self._ring.append(_Window(torch.empty(window_bytes, dtype=torch.uint8, pin_memory=True)))
        self._arena = arena
        self._next = 0
        self._copy_stream = torch.cuda.Stream(device)
        self._windows_pool = ThreadPoolExecutor(offload_workers, thread_name_prefix="ts-offload")
        self._slices_pool = ThreadPoolExecutor(reduction_workers, thread_name_prefix="ts-reduce")
        self._splits = reduction_workers
        self._lock = threading.Lock()
        self._staging: torch.Tensor | None = None
        self.report = {"folds": 0, "fold_bytes": 0, "combines": 0, "combine_bytes": 0, "windows": windows,
                       "window_bytes": window_bytes, "offload_workers": offload_workers,
                       "reduction_workers": reduction_workers, "arena_windows": arena is not None}

    # ------------------------------------------------------------ helpers
    def _take(self) -> _Window:
        w = self._ring[self._next]
        self._next = (self._next + 1) % len(self._ring)
        for f in w.pending:  # the window's previous host work must be done before it is reused
            f.result()
        w.pending = []
        if w.copied is not None:
            w.copied.synchronize()
        return w

    def _split(self, fn, n: int) -> None:
        """Run ``fn(lo, hi)`` over ``reduction_workers`` slices of [0, n) and wait for them."""
        step = -(-n // self._splits)
        futs = [self._slices_pool.submit(fn, lo, min(n, lo + step)) for lo in range(0, n, step)]
        for f in futs:
            f.result()

    # ------------------------------------------------------------ device -> host
    def fold(self, src: torch.Tensor, g1: torch.Tensor | None, g2: torch.Tensor | None, r: float) -> None:
        """``g1 += r·src`` (skipped when ``g1`` is None or r == 0) and ``g2 += src`` (skipped when None).

        ``src`` is a contiguous fp32 CUDA vector; ``g1``/``g2`` host vectors of the same length. Returns once
        every copy is enqueued; the caller's stream waits for the copies (so ``src`` may be overwritten by
        later stream work), the host adds run in the background until :meth:`drain`.
        """
        if src.dtype != torch.float32 or not src.is_cuda or not src.is_contiguous():
            raise ValueError("host fold sources are contiguous fp32 CUDA vectors")
        main = torch.cuda.current_stream(self.device)
        self._copy_stream.wait_stream(main)
        n = src.numel()
        for lo in range(0, n, self.window_elems):
            hi = min(n, lo + self.window_elems)
            w = self._take()
            host = w.buf.view(torch.float32)[: hi - lo]
            with torch.cuda.stream(self._copy_stream):
                host.copy_(src[lo:hi], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self._copy_stream)
            w.copied = ev

            def add(ev=ev, host=host, lo=lo, hi=hi):
                ev.synchronize()

                def part(a, b):
                    chunk = host[a:b]
                    if g2 is not None:
                        g2[lo + a : lo + b].add_(chunk.to(g2.dtype))
                    if g1 is not None and r != 0.0:
                        g1[lo + a : lo + b].add_(chunk.to(g1.dtype), alpha=r)

                self._split(part, hi - lo)

            w.pending.append(self._windows_pool.submit(add))
        main.wait_stream(self._copy_stream)
        with self._lock:
            self.report["folds"] += 1
            self.report["fold_bytes"] += 4 * n

    def pending(self) -> bool:
        """Whether host folds are still running (nothing waits)."""
        return self.pending_count() > 0

    def pending_count(self) -> int:
        """Host window folds and combines still running."""
        return sum(1 for w in self._ring for f in w.pending if not f.done())

    def drain(self) -> None:
        """Wait for every host fold and combine still running."""
        for w in self._ring:
            for f in w.pending:
                f.result()
            w.pending = []

    # ------------------------------------------------------------ host -> device
    def combine_into(self, out: torch.Tensor, g1: torch.Tensor, g2: torch.Tensor | None, a: float,
                     b: float) -> None:
        """``out += a·g1 + b·g2`` for a contiguous fp32 CUDA ``out`` and host ``g1``/``g2`` (``g2`` may be
        None); enqueued on the caller's stream."""
        from thundersync_b200.ops.fold import axpby_

        self.drain()
        main = torch.cuda.current_stream(self.device)
        n = out.numel()
        if self._staging is None or self._staging.numel() < self.window_elems * len(self._ring):
            self._staging = torch.empty(self.window_elems * len(self._ring), dtype=torch.float32, device=self.device)
        for k, lo in enumerate(range(0, n, self.window_elems)):
            hi = min(n, lo + self.window_elems)
            slot = self._next
            w = self._take()
            host = w.buf.view(torch.float32)[: hi - lo]

            def mix(x, y, lo=lo, host=host):
                seg = g1[lo + x : lo + y].to(torch.float32)
                torch.mul(seg, a, out=host[x:y])
                if g2 is not None:
                    host[x:y].add_(g2[lo + x : lo + y].to(torch.float32), alpha=b)

            self._split(mix, hi - lo)
            stage = self._staging[slot * self.window_elems : slot * self.window_elems + (hi - lo)]
            stage.copy_(host, non_blocking=True)  # H2D on the caller's stream, ordered before the add
            axpby_(out[lo:hi], stage, None, 1.0)
            ev = torch.cuda.Event()
            ev.record(main)
            w.copied = ev  # the window may be rewritten only after this copy has read it
        with self._lock:
            self.report["combines"] += 1
            self.report["combine_bytes"] += 4 * n

    _shared: dict[tuple, "HostFoldPipeline"] = {}
    _shared_lock = threading.Lock()

    @classmethod
    def shared(cls, device: torch.device, **options: Any) -> "HostFoldPipeline":
        """One pipeline per device and option set, reused across batches (its page-locked windows cost
        ~100 ms each to register); pipelines with a pinned arena are never shared."""
        if options.get("arena") is not None:
            return cls(device, **options)
        key = (str(device), tuple(sorted(options.items())))
        with cls._shared_lock:
            pipe = cls._shared.get(key)
            if pipe is None or not pipe._ring:
                pipe = cls._shared[key] = cls(device, **options)
            return pipe

    def close(self) -> None:
        self.drain()
        for w in self._ring:
            if w.copied is not None:
                w.copied.synchronize()
            if w.slab is not None and self._arena is not None:
                self._arena.release(w.slab)
        self._ring = []
        self._windows_pool.shutdown(wait=True)
        self._slices_pool.shutdown(wait=True)
