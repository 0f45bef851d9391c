"""Token embedding lookup whose weight gradient honours the gradient sink.

The backward is a deterministic sorted segment sum on CUDA (native kernel:
rows are grouped by token id and each output row is written by exactly one
CTA, in ascending source order) and ``index_add_`` on CPU.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops._ext import native


class _Embedding(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, weight):
        ctx.save_for_backward(ids)
        ctx.weight = weight
        return weight.index_select(0, ids)

    @staticmethod
    def backward(ctx, dy):
        (ids,) = ctx.saved_tensors
        weight = ctx.weight
        ctx.weight = None
        if not ctx.needs_input_grad[1]:
            return None, None
        s = _sink.active()
        target = s.view(weight) if (s is not None and s.owns(weight)) else None
        if target is None:
            target = torch.zeros(weight.shape, dtype=torch.float32, device=weight.device)
            out = target
        else:
            out = None
        scale = s.scale if (s is not None and out is None) else 1.0
        dy = dy.contiguous()
        if dy.is_cuda:
            native().embedding_bwd_accumulate(target, ids.contiguous(), dy, float(scale))
        else:
            target.index_add_(0, ids, dy.float(), alpha=scale)
        if out is None:
            s.deposits += 1
            return None, None
        return None, out.to(weight.dtype)


def embedding(ids: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    return _Embedding.apply(ids, weight)
