"""LoRA projection (K11′): ``y = x·Wᵀ + s·(x·Aᵀ)·Bᵀ`` without merging B·A into W.

The frozen base weight W keeps its dtype (bf16); the adapters A [r, in] and
B [out, r] are fp32 parameters. On CUDA with bf16 activations every product
is this package's tcgen05 GEMM with fp32 accumulation (the adapters are read
as bf16, as a bf16 PEFT forward reads them) and the base product enters the
rank-r GEMM's epilogue, so the output is rounded once; elsewhere the
low-rank path runs in fp32 — the numerics of an unmerged PEFT ``lora.Linear``
(reference: src/thundersync/policy_model.py:240-290 builds it through PEFT).

The reference's fused variant (src/thundersync/accel/fused_lora.py:26-50)
merges B·A into W in place for one forward GEMM and must unmerge before every
optimizer step. This op needs neither: the rank-r products are two thin
GEMMs beside the base GEMM, their fp32 weight gradients go straight into the
active gradient sink (``dA += s·(dy·B)ᵀ·x``, ``dB += s·dyᵀ·(x·Aᵀ)``), and
the frozen base never receives a gradient. Saved state is x plus the
[T, r] projection ``x·Aᵀ`` (fp32 on the CPU path; s·x·Aᵀ in bf16 on CUDA).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops.gemm import gemm

__all__ = ["lora_linear", "lora_parts"]


def lora_parts(mod: torch.nn.Module, adapter: str = "default"):
    """(base weight, A, B, scaling) of a PEFT-layout LoRA module."""
    a = mod.lora_A[adapter].weight if isinstance(mod.lora_A, torch.nn.ModuleDict) else mod.lora_A.weight
    b = mod.lora_B[adapter].weight if isinstance(mod.lora_B, torch.nn.ModuleDict) else mod.lora_B.weight
    sc = mod.scaling[adapter] if isinstance(mod.scaling, dict) else float(mod.scaling)
    return mod.base_layer.weight, a, b, float(sc)


def _deposit(param: torch.Tensor, lhs: torch.Tensor, rhs: torch.Tensor):
    """``lhsᵀ·rhs`` into the active sink when it owns ``param``; else return it (fp32-accumulated)."""
    s = _sink.active()
    if s is not None and s.owns(param):
        s.addmm_(s.view(param), lhs, rhs)
        return None
    if lhs.is_cuda and lhs.dtype == torch.bfloat16:
        return gemm(lhs, rhs, a_t=True, b_t=False, out_dtype=torch.float32).to(param.dtype)
    return lhs.t().matmul(rhs).to(param.dtype)


def _tc(x: torch.Tensor) -> bool:
    """CUDA bf16 activations: the rank-r products run as bf16 tensor-core GEMMs with fp32 accumulation."""
    return x.is_cuda and x.dtype == torch.bfloat16


# CUDA: the base product and the rank-r update run as ONE tcgen05 GEMM whose main loop continues over a
# second operand pair (y = x·Wᵀ + (s·u)·Bᵀ, dx = dy·W + (s·g)·A); False: library GEMMs
FUSED_TC = True


def _fused_ok(w: torch.Tensor, r: int) -> bool:
    return FUSED_TC and w.shape[0] % 64 == 0 and w.shape[1] % 64 == 0 and r % 8 == 0 and w.is_contiguous()


_BF16: dict[int, tuple] = {}


def _bf16_scaled(p: torch.Tensor, scale: float, dtype: torch.dtype) -> torch.Tensor:
    """``(scale · p)`` in the activation dtype, reused until ``p`` changes (its version counter moves at
    every in-place update, i.e. at each optimizer step)."""
    key = id(p)
    hit = _BF16.get(key)
    stamp = (p._version, p.data_ptr(), scale, dtype)
    if hit is not None and hit[0] == stamp:
        return hit[1]
    with torch.no_grad():
        t = (p.detach() * scale).to(dtype).contiguous() if scale != 1.0 else p.detach().to(dtype).contiguous()
    if len(_BF16) > 4096:
        _BF16.clear()
    _BF16[key] = (stamp, t)
    return t


class _LoRALinear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, a, b, scale):
        x2 = x.reshape(-1, x.shape[-1])
        if _tc(x2):
            # u = s·x·Aᵀ (fp32 accumulation, bf16 result, saved for dB); with the fused GEMM the rank-r
            # update is the main loop's last K block, otherwise the base product is the C operand of the
            # rank-r GEMM: either way y is rounded once
            u = gemm(x2, _bf16_scaled(a, scale, x2.dtype))
            bb = _bf16_scaled(b, 1.0, x2.dtype)
            if _fused_ok(w, a.shape[0]):
                from thundersync_b200.ops._ext import native

                y = x2.new_empty(x2.shape[0], w.shape[0])
                native().gemm_tc_cat(y, x2.contiguous(), w, u, bb, False, True, 0, 1.0)
            else:
                y = gemm(u, bb, residual=gemm(x2, w))
        else:
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
        dx = da = db = dw = None
        if _tc(dy2):
            ab = _bf16_scaled(a, 1.0, dy2.dtype)
            gs = gemm(dy2, _bf16_scaled(b, s, dy2.dtype), b_t=False)  # s·dy·B [T, r]
            if ctx.needs_input_grad[0]:
                if _fused_ok(w, a.shape[0]):
                    from thundersync_b200.ops._ext import native

                    dx = dy2.new_empty(dy2.shape[0], w.shape[1])
                    native().gemm_tc_cat(dx, dy2.contiguous(), w, gs, ab.contiguous(), False, False, 0, 1.0)
                    dx = dx.view(ctx.in_shape)
                else:
                    dx = gemm(gs, ab, b_t=False, residual=gemm(dy2, w, b_t=False)).view(ctx.in_shape)
            if ctx.needs_input_grad[2]:
                da = _deposit(a, gs, x2)
            if ctx.needs_input_grad[3]:
                db = _deposit(b, dy2, u)  # u already carries s
        else:
            dyf = dy2.to(b.dtype)
            g = dyf.matmul(b)  # [T, r]
            if ctx.needs_input_grad[0]:
                dx = torch.addmm(dy2.matmul(w).to(g.dtype), g, a, alpha=s).to(x2.dtype).view(ctx.in_shape)
            if ctx.needs_input_grad[2]:
                da = _deposit(a, g * s, x2.to(a.dtype))
            if ctx.needs_input_grad[3]:
                db = _deposit(b, dyf, u * s)
        if ctx.needs_input_grad[1]:
            dw = gemm(dy2, x2, a_t=True, b_t=False, out_dtype=torch.float32).to(w.dtype)
        return dx, dw, da, db, None


def lora_linear(x: torch.Tensor, mod: torch.nn.Module, adapter: str = "default") -> torch.Tensor:
    """``mod(x)`` for a PEFT-layout LoRA module (``base_layer`` + ``lora_A``/``lora_B``)."""
    w, a, b, s = lora_parts(mod, adapter)
    if getattr(mod, "_thundersync_fused", False):  # merged-weight mode (accel.fused_lora)
        from thundersync_b200.accel.fused_lora import FusedLoRALinear

        return FusedLoRALinear.apply(x, w, a, b, s)
    return _LoRALinear.apply(x, w, a, b, s)
