"""Data-parallel gradient reduction of the flat fp32 batch gradient (N1/N2 host side).

``GradientReducer.all_reduce_mean(grad, pre_scale)`` leaves every rank with
``mean_over_ranks(pre_scale * grad)``. The flat buffer is reduced in buckets
so each collective is large enough to reach link bandwidth and the
reduction can start while later buckets are still being produced.

Transport: this package's NVLink kernels (``thundersync_b200.parallel.symm``)
when every rank of the group is a CUDA device on one node and the symmetric
buffers could be mapped; NCCL through ``torch.distributed`` otherwise (and on
CPU, gloo). The pre-scale is folded into the native kernel's load; on the
NCCL path it is one fused scale kernel before the collective.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from thundersync_b200.ops.fold import scale_

__all__ = ["GradientReducer"]

DEFAULT_BUCKET_ELEMS = 64 * 1024 * 1024  # 256 MiB of fp32


class GradientReducer:
    def __init__(self, numel: int, device: torch.device, *, bucket_elems: int = DEFAULT_BUCKET_ELEMS,
                 group=None, native: bool | None = None) -> None:
        self.numel = int(numel)
        self.device = device
        self.bucket_elems = int(bucket_elems)
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.native = None
        if native is not False and device.type == "cuda" and self.world > 1:
            try:
                from thundersync_b200.parallel.symm import NativeAllReduce

                self.native = NativeAllReduce.create(min(self.numel, self.bucket_elems), device, group)
            except Exception as exc:  # pragma: no cover - depends on the node
                if native:
                    raise
                self.native_error = repr(exc)
                self.native = None
        self.last_path = None

    def all_reduce_mean(self, grad: torch.Tensor, *, pre_scale: float = 1.0) -> None:
        if self.world == 1:
            if pre_scale != 1.0:
                scale_(grad, pre_scale)
            return
        if self.native is not None:
            self.native.all_reduce_mean(grad, pre_scale=pre_scale)
            self.last_path = "native"
            return
        s = pre_scale / self.world
        if s != 1.0:
            if grad.is_cuda:
                scale_(grad, s)
            else:
                grad.mul_(s)
        for lo in range(0, grad.numel(), self.bucket_elems):
            dist.all_reduce(grad[lo : lo + self.bucket_elems], op=dist.ReduceOp.SUM, group=self.group)
        self.last_path = "nccl" if grad.is_cuda else "gloo"

    def close(self) -> None:
        if self.native is not None:
            self.native.close()
            self.native = None
