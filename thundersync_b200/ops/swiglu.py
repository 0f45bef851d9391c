"""SwiGLU activation over the fused gate/up projection output [T, 2F].

``a = silu(g) · u`` with ``g = gu[:, :F]`` and ``u = gu[:, F:]``, fp32 math,
one rounding. The backward recomputes ``silu`` from ``gu``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from thundersync_b200.ops._ext import native


def swiglu_reference(gu: torch.Tensor) -> torch.Tensor:
    f = gu.shape[-1] // 2
    g, u = gu[..., :f].float(), gu[..., f:].float()
    return (F.silu(g) * u).to(gu.dtype)


class _SwiGLU(torch.autograd.Function):
    @staticmethod
    def forward(ctx, gu):
        ctx.save_for_backward(gu)
        if gu.is_cuda:
            return native().swiglu_fwd(gu.contiguous())
        return swiglu_reference(gu)

    @staticmethod
    def backward(ctx, da):
        (gu,) = ctx.saved_tensors
        if gu.is_cuda:
            return native().swiglu_bwd(da.contiguous(), gu.contiguous())
        f = gu.shape[-1] // 2
        g, u = gu[..., :f].float(), gu[..., f:].float()
        sg = torch.sigmoid(g)
        silu = g * sg
        dg = da.float() * u * (sg * (1 + g * (1 - sg)))
        du = da.float() * silu
        return torch.cat((dg, du), -1).to(gu.dtype)


def swiglu(gu: torch.Tensor) -> torch.Tensor:
    return _SwiGLU.apply(gu)
