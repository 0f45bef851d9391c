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


def _ref_forward(x2: torch.Tensor, w: torch.Tensor, eps: float, unit: bool = False):
    xf = x2.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1) + eps)
    if unit:
        return (xf * rstd[:, None] * (1.0 + w.float())).to(x2.dtype), rstd
    n = (xf * rstd[:, None]).to(x2.dtype)
    y = (w.float() * n.float()).to(x2.dtype)
    return y, rstd


def _ref_backward(dy2, x2, w, rstd, unit: bool = False):
    n = x2.float() * rstd[:, None]
    dn = dy2.float() * (w.float() + 1.0 if unit else w.float())
    dx = rstd[:, None] * (dn - n * (dn * n).mean(-1, keepdim=True))
    dw = (dy2.float() * n).sum(0)
    return dx.to(x2.dtype), dw


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps, unit):
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if x2.is_cuda:
            y, rstd = native().rms_norm_fwd(x2, w.contiguous(), float(eps), bool(unit))
        else:
            y, rstd = _ref_forward(x2, w, eps, unit)
        ctx.save_for_backward(x2, w, rstd)
        ctx.shape = shape
        ctx.unit = unit
        return y.view(shape)

    @staticmethod
    def backward(ctx, dy):
        return _RMSNorm.backward_residual(ctx, dy, None)

    @staticmethod
    def backward_residual(ctx, dy, dres):
        """The VJP with ``dres`` (a residual branch's gradient, shaped like x) added to dx; on CUDA the add is
        fused into the kernel before the single rounding of dx."""
        x2, w, rstd = ctx.saved_tensors
        dy2 = dy.reshape(x2.shape)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        s = _sink.active() if ctx.needs_input_grad[1] else None
        into_sink = s is not None and s.owns(w)
        if dy2.is_cuda:
            r2 = None if dres is None else dres.reshape(x2.shape).contiguous()
            # a sink-owned weight's gradient is summed straight into the sink by the kernel's final reduction
            acc = s.view(w) if into_sink and s.view(w).dtype == torch.float32 else None
            dx, dw = native().rms_norm_bwd(dy2, x2, w.contiguous(), rstd, bool(ctx.unit), r2, acc,
                                           float(s.scale) if acc is not None else 1.0)
            if acc is not None:
                s.deposits += 1
                into_sink = False
                dw = None
        else:
            dx, dw = _ref_backward(dy2, x2, w, rstd, ctx.unit)
            if dres is not None:
                dx = dres.reshape(dx.shape) + dx
        dw_out = None
        if into_sink:
            s.add_(w, dw)
        elif ctx.needs_input_grad[1] and dw is not None and not (s is not None and s.owns(w)):
            dw_out = dw.to(w.dtype)
        return dx.view(ctx.shape), dw_out, None, None


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float, unit_offset: bool = False) -> torch.Tensor:
    """``unit_offset``: the weight is stored zero-centred and applied as ``1 + w``
    with a single fp32 rounding (Qwen3.5 convention)."""
    return _RMSNorm.apply(x, weight, eps, unit_offset)


def rms_norm_reference(x: torch.Tensor, weight: torch.Tensor, eps: float, unit_offset: bool = False) -> torch.Tensor:
    """Differentiable plain-torch oracle (fp32 math, same roundings)."""
    xf = x.float()
    r = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if unit_offset:
        return (xf * r * (1.0 + weight.float())).to(x.dtype)
    n = (xf * r).to(x.dtype)
    return (weight.float() * n.float()).to(x.dtype)
