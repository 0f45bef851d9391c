"""RMSNorm forward/backward (K12′): native row kernels on CUDA, fp32 torch on CPU.

Semantics follow Qwen3's RMSNorm: ``y = w · cast(x·rstd)`` with
``rstd = rsqrt(mean(x²) + eps)`` computed in fp32 and the normalised value
rounded to the input dtype before the weight multiply. The VJP is computed in
fp32 (reference: src/thundersync/accel/rms_norm.py:7-43, K12/K13): the weight
gradient is reduced in a fixed order (per-CTA partials, then one ordered
sum), so it is deterministic without atomics.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops._ext import native


def _ref_forward(x2: torch.Tensor, w: torch.Tensor, eps: float):
    xf = x2.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    n = (xf * rstd[:, None]).to(x2.dtype)
    y = (w.float() * n.float()).to(x2.dtype)
    return y, rstd


def _ref_backward(dy2, x2, w, rstd):
    n = x2.float() * rstd[:, None]
    dn = dy2.float() * w.float()
    dx = rstd[:, None] * (dn - n * (dn * n).mean(-1, keepdim=True))
    dw = (dy2.float() * n).sum(0)
    return dx.to(x2.dtype), dw


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if x2.is_cuda:
            y, rstd = native().rms_norm_fwd(x2, w.contiguous(), float(eps))
        else:
            y, rstd = _ref_forward(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        if dy2.is_cuda:
            dx, dw = native().rms_norm_bwd(dy2, x2, w.contiguous(), rstd)
        else:
            dx, dw = _ref_backward(dy2, x2, w, rstd)
        dw_out = None
        if ctx.needs_input_grad[1]:
            s = _sink.active()
            if s is not None and s.owns(w):
                s.add_(w, dw)
            else:
                dw_out = dw.to(w.dtype)
        return dx.view(ctx.shape), dw_out, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return _RMSNorm.apply(x, weight, eps)


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Differentiable plain-torch oracle (fp32 math, same roundings)."""
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return (weight.float() * n.float()).to(x.dtype)
