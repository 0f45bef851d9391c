"""Per-parameter data-parallel gradient average (C38).

One asynchronous ``all_reduce`` per parameter gradient, then a wait on all of
them: the collective order is the parameter order, identical on every rank
(reference: src/thundersync/grpo/gradient_average.py:9-25). ``AVG`` is
expressed as SUM then a scale by 1/world, which every backend supports.

This is the generic path for gradients held per parameter. The GRPO
data-parallel trainer keeps its gradient in one flat fp32 buffer and averages
it with this package's peer-memory reduction (or one flat NCCL call), see
:mod:`thundersync_b200.parallel.reduce`.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

__all__ = ["per_parameter_all_reduce_average"]


def per_parameter_all_reduce_average(parameters: list[torch.nn.Parameter]) -> dict[str, int | str]:
    world = dist.get_world_size()
    handles = [dist.all_reduce(p.grad, op=dist.ReduceOp.SUM, async_op=True) for p in parameters]
    for h in handles:
        h.wait()
    for p in parameters:
        p.grad.div_(world)
    return {"allreduce_mode": "per_parameter_async", "allreduce_collectives": len(handles),
            "allreduce_bucket_cap_bytes": 0, "allreduce_peak_bucket_bytes": 0}
