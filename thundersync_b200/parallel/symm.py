"""Peer-mapped workspace and the native NVLink collectives (N0-N3, host side).

Buffers are dedicated ``cudaMalloc`` allocations exported with CUDA IPC
handles; the handles are exchanged through the process group and every peer
opens them, so each rank holds device pointers to every rank's buffer
(``csrc/ipc.cpp``; plain peer mappings, no multicast objects). Every
collective is this package's kernel (``csrc/comm.cu``) reading and writing
peer memory over NVLink:

* ``barrier``            bounded-wait flag barrier; a peer that never arrives
                         sets a device status word instead of hanging
                         (``check()`` raises :class:`CollectiveTimeout`);
* ``all_reduce_mean``    in-place deterministic two-shot all-reduce of a flat
                         fp32 buffer with the pre-scale fused into the load;
* ``all_reduce_mean_oneshot``  every rank reads every rank's whole buffer
                         and writes the mean to a local output: one NVLink
                         phase instead of two, for buffers below
                         ``oneshot_max_elems(world)`` (latency-bound sizes);
* ``reduce_scatter``     the first half only, plus the squared norm of each
                         reduced shard exchanged through the flag buffer;
* ``adamw_gather``       fused AdamW on this rank's shard that writes the
                         bf16 parameters straight into every rank's
                         parameter buffer (ZeRO-1 all-gather fused with the
                         fp32->bf16 cast).

All reductions sum ranks in a fixed order, so every rank holds bitwise
identical results. No TMA multicast is used anywhere.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from thundersync_b200.ops._ext import native

__all__ = ["SymmetricWorkspace", "NativeAllReduce", "CollectiveTimeout", "shard_bounds", "ONESHOT_MAX_ELEMS",
           "oneshot_max_elems"]

# Crossover between the one-shot and the two-shot all-reduce, in fp32 elements per rank count. Below it
# the second barrier-separated phase of the two-shot costs more than the extra (world - 1) / world of the
# buffer each rank reads in the one-shot. Measured on two B200s (benchmarks/bench_collectives.py): the
# one-shot is faster through 16 MiB (0.050 vs 0.052 ms) and slower at 256 MiB (0.443 vs 0.422 ms); the
# one-shot's read volume grows with the world size, so the threshold scales as 1 / world.
ONESHOT_MAX_BYTES_X_WORLD = 32 << 20


def oneshot_max_elems(world: int) -> int:
    return ONESHOT_MAX_BYTES_X_WORLD // (4 * max(1, world))


ONESHOT_MAX_ELEMS = oneshot_max_elems(2)

_SLOTS = 64
_MAX_RANKS = 8
_NORM_OFFSET = _SLOTS * _MAX_RANKS  # u32 index where the fp32 norm slots start


class CollectiveTimeout(RuntimeError):
    """A device-side wait ran out: the named peer never arrived."""


def shard_bounds(numel: int, world: int, rank: int, align: int = 4) -> tuple[int, int]:
    chunk = -(-numel // world)
    chunk = -(-chunk // align) * align
    lo = min(numel, rank * chunk)
    return lo, min(numel, lo + chunk)


class SymmetricWorkspace:
    """Peer-mapped buffers of one process group on this rank's device."""

    def __init__(self, device: torch.device, group=None, *, timeout_s: float = 30.0) -> None:
        self.device = device
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > _MAX_RANKS:
            raise ValueError(f"the native collectives support up to {_MAX_RANKS} ranks")
        self.timeout_s = float(timeout_s)
        self._owned: list[torch.Tensor] = []
        self._opened: list[int] = []
        self.flags, self.flag_ptrs = self.alloc(_NORM_OFFSET + _MAX_RANKS, torch.int32)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        self._epochs = [0] * _SLOTS
        torch.cuda.synchronize(device)
        dist.barrier(group)

    def alloc(self, numel: int, dtype: torch.dtype) -> tuple[torch.Tensor, list[int]]:
        """A zeroed buffer on every rank; returns (local tensor, every rank's device pointer)."""
        esize = torch.empty(0, dtype=dtype).element_size()
        nbytes = -(-numel * esize // 256) * 256
        raw, handle = native().ipc_alloc(nbytes, self.device.index)
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=self.group)
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(int(raw.data_ptr()))
            else:
                p = int(native().ipc_open(h, self.device.index))
                self._opened.append(p)
                ptrs.append(p)
        self._owned.append(raw)
        t = raw.view(dtype)[:numel]
        return t, ptrs

    @property
    def norm_slots(self) -> torch.Tensor:
        return self.flags[_NORM_OFFSET : _NORM_OFFSET + self.world].view(torch.float32)

    def barrier(self, slot: int = 0) -> None:
        self._epochs[slot] += 1
        native().symm_barrier(self.flag_ptrs, self.rank, slot, self._epochs[slot], self.status, self.timeout_s)

    def check(self) -> None:
        code = int(self.status.item())
        if code:
            raise CollectiveTimeout(
                f"rank {self.rank}: native collective wait expired waiting for rank {code - 1000} "
                f"(timeout {self.timeout_s} s)"
            )

    def all_reduce_mean(self, buf: torch.Tensor, ptrs: list[int], *, pre_scale: float = 1.0) -> None:
        """In place: ``buf`` (symmetric fp32) becomes mean over ranks of ``pre_scale * buf``."""
        lo, hi = shard_bounds(buf.numel(), self.world, self.rank)
        self.barrier(0)
        native().symm_reduce(ptrs, self.rank, lo, hi, pre_scale / self.world, True, buf)
        self.barrier(1)

    def all_reduce_mean_oneshot(self, buf: torch.Tensor, ptrs: list[int], out: torch.Tensor, *,
                                pre_scale: float = 1.0) -> None:
        """``out`` (local, contiguous fp32) becomes the mean over ranks of ``pre_scale * buf``; ``buf`` is
        left as it was. The closing barrier keeps ``buf`` unchanged until every peer has read it."""
        self.barrier(0)
        native().symm_reduce_oneshot(ptrs, buf.numel(), pre_scale / self.world, out)
        self.barrier(1)

    def reduce_scatter(self, buf: torch.Tensor, ptrs: list[int], *, pre_scale: float = 1.0) -> tuple[int, int]:
        """This rank's shard of ``buf`` becomes the mean; its squared norm goes to every rank's slot."""
        lo, hi = shard_bounds(buf.numel(), self.world, self.rank)
        self.barrier(0)
        partial = native().symm_reduce(ptrs, self.rank, lo, hi, pre_scale / self.world, False, buf)
        native().symm_norm_put(partial, self.flag_ptrs, self.rank, _NORM_OFFSET)
        self.barrier(1)
        return lo, hi

    def close(self) -> None:
        """Unmap peers, wait for every rank to do the same, then free local buffers."""
        if self.flags is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            native().ipc_close(p)
        self._opened.clear()
        if dist.is_initialized():
            dist.barrier(self.group)
        self._owned.clear()
        self.flags = None


class NativeAllReduce:
    """All-reduce of a caller's (non-symmetric) flat fp32 buffer through a symmetric bucket."""

    def __init__(self, ws: SymmetricWorkspace, bucket_elems: int) -> None:
        self.ws = ws
        self.bucket_elems = -(-bucket_elems // (4 * ws.world)) * 4 * ws.world
        self.bucket, self.ptrs = ws.alloc(self.bucket_elems, torch.float32)

    @classmethod
    def create(cls, bucket_elems: int, device: torch.device, group=None) -> "NativeAllReduce":
        return cls(SymmetricWorkspace(device, group), bucket_elems)

    def all_reduce_mean(self, grad: torch.Tensor, *, pre_scale: float = 1.0, oneshot: bool | None = None) -> None:
        """Mean over ranks of ``pre_scale * grad``, in place; one-shot below ``ONESHOT_MAX_ELEMS`` elements
        (``oneshot`` forces either algorithm)."""
        n = grad.numel()
        if oneshot is None:
            oneshot = n <= oneshot_max_elems(self.ws.world)
        if oneshot and n <= self.bucket_elems and grad.is_contiguous() and grad.data_ptr() % 16 == 0:
            view = self.bucket[:n]
            view.copy_(grad)
            self.ws.all_reduce_mean_oneshot(view, self.ptrs, grad, pre_scale=pre_scale)
            self.ws.check()
            return
        b = self.bucket_elems
        for lo in range(0, n, b):
            hi = min(n, lo + b)
            view = self.bucket[: hi - lo]
            view.copy_(grad[lo:hi])
            if hi - lo < b:
                self.bucket[hi - lo :].zero_()
            self.ws.all_reduce_mean(self.bucket, self.ptrs, pre_scale=pre_scale)
            grad[lo:hi].copy_(view)
        self.ws.check()

    def close(self) -> None:
        self.ws.close()
