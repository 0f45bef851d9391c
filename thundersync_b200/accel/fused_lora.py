"""Merged-weight LoRA forward, for callers that want the reference's fused mode.

``fuse_merged_lora_forward`` merges ``s·B·A`` into each adapted layer's base
weight in place and routes the layer through :class:`FusedLoRALinear` — one
GEMM forward, with the adapter gradients from rank-sized GEMMs in the
backward (``dx = g·W_eff``, ``dA = s·(g·B)ᵀ·x``, ``dB = s·gᵀ·(x·Aᵀ)``);
``unfuse_merged_lora_forward`` restores the base weight and the stock
forward and must run before every optimizer step (reference:
src/thundersync/accel/fused_lora.py:26-126).

This framework's default LoRA forward (:func:`thundersync_b200.ops.lora.lora_linear`)
needs no merge at all; this module exists so a configuration with
``fused_lora=True`` behaves as it did.
"""

from __future__ import annotations

import torch

__all__ = ["FusedLoRALinear", "fuse_merged_lora_forward", "unfuse_merged_lora_forward"]


class FusedLoRALinear(torch.autograd.Function):
    """``x @ W_effᵀ`` with adapter gradients; no adapter GEMM in the forward."""

    @staticmethod
    def forward(ctx, x, weight, lora_a, lora_b, scaling):
        ctx.save_for_backward(x, weight, lora_a, lora_b)
        ctx.scaling = scaling
        return x @ weight.t()

    @staticmethod
    def backward(ctx, g):
        x, weight, lora_a, lora_b = ctx.saved_tensors
        s = ctx.scaling
        a, b = lora_a.to(x.dtype), lora_b.to(x.dtype)
        dx = g @ weight
        da = db = None
        if ctx.needs_input_grad[2]:
            da = ((g @ b).transpose(-2, -1) @ x * s).to(lora_a.dtype)
        if ctx.needs_input_grad[3]:
            db = (g.transpose(-2, -1) @ (x @ a.t()) * s).to(lora_b.dtype)
        return dx, None, da, db, None


def _active(model: torch.nn.Module) -> str:
    adapter = getattr(model, "active_adapter", "default")
    if isinstance(adapter, (list, tuple)):
        if len(adapter) != 1:
            raise ValueError("fused LoRA supports one active adapter")
        adapter = adapter[0]
    return adapter


def fuse_merged_lora_forward(peft_model: torch.nn.Module) -> int:
    """Merge adapters into base weights in place and route through the fused path; returns layers converted."""
    from thundersync_b200.models.lora import LoRALinear

    adapter = _active(peft_model)
    n = 0
    for m in peft_model.modules():
        if not isinstance(m, LoRALinear) or getattr(m, "_thundersync_fused", False):
            continue
        a, b, s = m.lora_A[adapter].weight, m.lora_B[adapter].weight, m.scaling[adapter]
        with torch.no_grad():
            w = m.base_layer.weight
            w.copy_((w.float() + s * (b.float() @ a.float())).to(w.dtype))

        def forward(x, _m=m, _a=a, _b=b, _s=s):
            return FusedLoRALinear.apply(x, _m.base_layer.weight, _a, _b, _s)

        m._thundersync_unfused_forward = m.forward
        m._thundersync_merge = (a.detach().clone(), b.detach().clone(), s)
        m.forward = forward
        m._thundersync_fused = True
        n += 1
    return n


def unfuse_merged_lora_forward(peft_model: torch.nn.Module) -> int:
    """Subtract the merged adapters (as merged) and restore the stock forward; returns layers restored."""
    n = 0
    for m in peft_model.modules():
        if not getattr(m, "_thundersync_fused", False):
            continue
        a, b, s = m._thundersync_merge
        with torch.no_grad():
            w = m.base_layer.weight
            w.copy_((w.float() - s * (b.float() @ a.float())).to(w.dtype))
        m.forward = m._thundersync_unfused_forward
        del m._thundersync_unfused_forward, m._thundersync_merge
        m._thundersync_fused = False
        n += 1
    return n
