"""Projection GEMMs with gradient-sink-aware weight gradients.

On CUDA every projection product (``y = x·Wᵀ [+ residual]``, ``dx = dy·W``,
``dW += dyᵀ·x``) runs on this package's tcgen05 GEMM (``ops/gemm.py``). Under
an active :class:`~thundersync_b200.ops.sink.GradSink` the backward
accumulates ``dW += dYᵀ·X`` straight into the sink's fp32 buffer (the GEMM
epilogue's TMA reduce-add), so no per-call weight gradient is ever allocated.
Several weights that sit back to back in the parameter arena (q/k/v,
gate/up) run as one GEMM over a single weight view.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops.gemm import gemm, matmul


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, fused, *weights):
        return _Linear.forward_residual(ctx, x, fused, None, *weights)

    @staticmethod
    def forward_residual(ctx, x, fused, residual, *weights):
        """``residual + x @ Wᵀ``; on CUDA the add is the GEMM's C operand (one rounding, no separate kernel)."""
        if fused is not None:
            w = fused
        elif len(weights) == 1:
            w = weights[0]
        else:
            w = torch.cat(weights, 0)
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1])
        r2 = None if residual is None else residual.reshape(-1, residual.shape[-1])
        y = gemm(x2, w, residual=r2).reshape(*lead, w.shape[0])
        ctx.save_for_backward(x, w)
        ctx.n_weights = len(weights)
        ctx.rows = [t.shape[0] for t in weights]
        ctx.weights = weights  # parameter identity for the sink (no storage held beyond w)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        weights = ctx.weights
        dx = None
        if ctx.needs_input_grad[0]:
            dx = matmul(dy, w)
        grads = [None] * ctx.n_weights
        need_w = any(ctx.needs_input_grad[2:])
        if need_w:
            dy2 = dy.reshape(-1, dy.shape[-1])
            x2 = x.reshape(-1, x.shape[-1])
            s = _sink.active()
            if s is not None and all(s.owns(t) for t in weights):
                # projection weights receive only this deposit: it may run on the side stream
                span = s.span_view(list(weights))
                if span is not None:
                    s.addmm_(span, dy2, x2, side=True)
                else:
                    r0 = 0
                    for t, r in zip(weights, ctx.rows):
                        s.addmm_(s.view(t), dy2[:, r0 : r0 + r], x2, side=True)
                        r0 += r
            else:
                dw = gemm(dy2, x2, a_t=True, b_t=False,
                          out_dtype=torch.float32 if dy2.is_cuda else dy2.dtype)
                r0 = 0
                for i, r in enumerate(ctx.rows):
                    if ctx.needs_input_grad[2 + i]:
                        grads[i] = dw[r0 : r0 + r].to(weights[i].dtype)
                    r0 += r
        ctx.weights = None
        return (dx, None, *grads)


def linear(x: torch.Tensor, weights: list[torch.Tensor] | torch.Tensor, arena=None) -> torch.Tensor:
    """``x @ cat(weights)ᵀ``; one GEMM over an arena view when the weights are adjacent."""
    if isinstance(weights, torch.Tensor):
        weights = [weights]
    fused = None
    if arena is not None and len(weights) > 1:
        fused = arena.fused_weight(list(weights))
    return _Linear.apply(x, fused, *weights)
