"""Data-parallel communication of the flat batch gradient and parameters (N1-N3, host side).

:class:`GradientReducer` owns the transport for one trainer:

* native (CUDA, one node, symmetric memory available): the batch gradient is
  itself a peer-mapped fp32 buffer, so the reduction runs in place with no
  copy -- a deterministic two-shot all-reduce for replicated optimizers, or a
  reduce-scatter followed by the fused AdamW + bf16 parameter all-gather for
  the sharded (ZeRO-1) optimizer, whose parameter arena is then peer-mapped
  too;
* otherwise NCCL (gloo on CPU) through ``torch.distributed``, in buckets.

``last_path`` records which one ran ("native", "nccl", "gloo").
"""

from __future__ import annotations

import logging

import torch
import torch.distributed as dist

from thundersync_b200.ops.fold import scale_

log = logging.getLogger(__name__)

__all__ = ["GradientReducer"]

DEFAULT_BUCKET_ELEMS = 64 * 1024 * 1024


class GradientReducer:
    def __init__(self, numel: int, device: torch.device, *, group=None, native: bool | None = None,
                 bucket_elems: int = DEFAULT_BUCKET_ELEMS, arena=None, shard_params: bool = False,
                 timeout_s: float = 30.0) -> None:
        self.numel = int(numel)
        self.device = device
        self.group = group
        self.bucket_elems = int(bucket_elems)
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.ws = None
        self.grad = None
        self.grad_ptrs: list[int] = []
        self.param_ptrs: list[int] = []
        self.native_error: str | None = None
        self.last_path: str | None = None
        if native is not False and device.type == "cuda" and self.world > 1:
            try:
                from thundersync_b200.parallel.symm import SymmetricWorkspace

                self.ws = SymmetricWorkspace(device, group, timeout_s=timeout_s)
                padded = -(-self.numel // (4 * self.world)) * 4 * self.world
                self.grad, self.grad_ptrs = self.ws.alloc(padded, torch.float32)
                self.grad.zero_()
                if shard_params and arena is not None:
                    flat, self.param_ptrs = self.ws.alloc(arena.numel, arena.dtype)
                    arena.rehome(flat)
                torch.cuda.synchronize(device)
                dist.barrier(group)
            except Exception as exc:  # pragma: no cover - depends on the node
                if native:
                    raise
                log.warning("native NVLink collectives unavailable, using NCCL: %r", exc)
                self.native_error = repr(exc)
                self.ws = None
                self.grad = None

    @property
    def native(self) -> bool:
        return self.ws is not None

    def main_grad_buffer(self) -> torch.Tensor | None:
        return self.grad

    def shard(self) -> tuple[int, int]:
        from thundersync_b200.parallel.symm import shard_bounds

        return shard_bounds(self.numel, self.world, self.rank)

    # ------------------------------------------------------------ replicated
    def all_reduce_mean(self, grad: torch.Tensor, *, pre_scale: float = 1.0) -> None:
        if self.world == 1:
            if pre_scale != 1.0:
                scale_(grad, pre_scale) if grad.is_cuda else grad.mul_(pre_scale)
            return
        if self.ws is not None and self.grad is not None and grad.data_ptr() == self.grad.data_ptr():
            self.ws.all_reduce_mean(self.grad, self.grad_ptrs, pre_scale=pre_scale)
            self.last_path = "native"
            return
        s = pre_scale / self.world
        if s != 1.0:
            scale_(grad, s) if grad.is_cuda else grad.mul_(s)
        for lo in range(0, grad.numel(), self.bucket_elems):
            dist.all_reduce(grad[lo : lo + self.bucket_elems], op=dist.ReduceOp.SUM, group=self.group)
        self.last_path = "nccl" if grad.is_cuda else "gloo"

    # ------------------------------------------------------------ sharded
    def reduce_scatter_mean(self, grad: torch.Tensor, *, pre_scale: float = 1.0) -> tuple[int, int]:
        """This rank's shard of ``grad`` becomes the mean (other shards are left unspecified)."""
        lo, hi = self.shard()
        if self.ws is not None and self.grad is not None and grad.data_ptr() == self.grad.data_ptr():
            self.ws.reduce_scatter(self.grad, self.grad_ptrs, pre_scale=pre_scale)
            self.last_path = "native"
            return lo, hi
        # NCCL: reduce-scatter over equal padded chunks
        self.all_reduce_mean(grad, pre_scale=pre_scale)
        return lo, hi

    def check(self) -> None:
        if self.ws is not None:
            self.ws.check()

    def close(self) -> None:
        if self.ws is not None:
            self.ws.close()
            self.ws = None
