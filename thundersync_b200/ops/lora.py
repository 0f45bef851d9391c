"""LoRA projection (K11′): ``y = x·Wᵀ + s·(x·Aᵀ)·Bᵀ`` without merging B·A into W.

The frozen base weight W keeps its dtype (bf16); the adapters A [r, in] and
B [out, r] are fp32 and so is the low-rank path, which is added to the bf16
base product before the single rounding to the activation dtype — the
numerics of an unmerged PEFT ``lora.Linear`` (reference:
src/thundersync/policy_model.py:240-290 builds it through PEFT).

The reference's fused variant (src/thundersync/accel/fused_lora.py:26-50)
merges B·A into W in place for one forward GEMM and must unmerge before every
optimizer step. This op needs neither: the rank-r products are two thin
GEMMs beside the base GEMM, their fp32 weight gradients go straight into the
active gradient sink (``dA += s·(dy·B)ᵀ·x``, ``dB += s·dyᵀ·(x·Aᵀ)``), and
the frozen base never receives a gradient. Saved state is x plus the
[T, r] fp32 projection ``x·Aᵀ``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from thundersync_b200.ops import sink as _sink

__all__ = ["lora_linear", "lora_parts"]


def lora_parts(mod: torch.nn.Module, adapter: str = "default"):
    """(base weight, A, B, scaling) of a PEFT-layout LoRA module."""
    a = mod.lora_A[adapter].weight if isinstance(mod.lora_A, torch.nn.ModuleDict) else mod.lora_A.weight
    b = mod.lora_B[adapter].weight if isinstance(mod.lora_B, torch.nn.ModuleDict) else mod.lora_B.weight
    sc = mod.scaling[adapter] if isinstance(mod.scaling, dict) else float(mod.scaling)
    return mod.base_layer.weight, a, b, float(sc)


def _deposit(param: torch.Tensor, lhs: torch.Tensor, rhs: torch.Tensor):
    """``lhsᵀ·rhs`` into the active sink when it owns ``param``; else return it."""
    s = _sink.active()
    if s is not None and s.owns(param):
        s.addmm_(s.view(param), lhs, rhs)
        return None
    return lhs.t().matmul(rhs).to(param.dtype)


class _LoRALinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, a, b, scale):
        x2 = x.reshape(-1, x.shape[-1])
        base = F.linear(x2, w)
        u = F.linear(x2.to(a.dtype), a)  # [T, r], adapter precision
        y = torch.addmm(base.to(u.dtype), u, b.t(), alpha=scale).to(x.dtype)
        ctx.save_for_backward(x2, w, a, b, u)
        ctx.scale = scale
        ctx.in_shape = x.shape
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w, a, b, u = ctx.saved_tensors
        s = ctx.scale
        dy2 = dy.reshape(-1, dy.shape[-1])
        dyf = dy2.to(b.dtype)
        g = dyf.matmul(b)  # [T, r]
        dx = da = db = dw = None
        if ctx.needs_input_grad[0]:
            dx = torch.addmm(dy2.matmul(w).to(g.dtype), g, a, alpha=s).to(x2.dtype).view(ctx.in_shape)
        if ctx.needs_input_grad[2]:
            da = _deposit(a, g * s, x2.to(a.dtype))
        if ctx.needs_input_grad[3]:
            db = _deposit(b, dyf, u * s)
        if ctx.needs_input_grad[1]:
            dw = dy2.t().matmul(x2).to(w.dtype)
        return dx, dw, da, db, None


def lora_linear(x: torch.Tensor, mod: torch.nn.Module, adapter: str = "default") -> torch.Tensor:
    """``mod(x)`` for a PEFT-layout LoRA module (``base_layer`` + ``lora_A``/``lora_B``)."""
    w, a, b, s = lora_parts(mod, adapter)
    if getattr(mod, "_thundersync_fused", False):  # merged-weight mode (accel.fused_lora)
        from thundersync_b200.accel.fused_lora import FusedLoRALinear

        return FusedLoRALinear.apply(x, w, a, b, s)
    return _LoRALinear.apply(x, w, a, b, s)
