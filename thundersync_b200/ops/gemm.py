"""tcgen05 GEMM (S4): ``out (op)= alpha · op(a) · op(b) [+ residual]`` in bf16 with fp32 accumulation.

``gemm(a, b, a_t=False, b_t=True)`` computes ``a @ b.T`` for an ``nn.Linear``
weight ``b`` [N, K]; ``b_t=False`` takes ``b`` as [K, N]; ``a_t=True`` takes
``a`` as [K, M]. So ``y = x·Wᵀ`` is ``gemm(x, W)``, ``dx = dy·W`` is
``gemm(dy, W, b_t=False)`` and ``dW = dyᵀ·x`` is ``gemm(dy, x, a_t=True,
b_t=False)`` — no transpose copies. ``residual`` adds a bf16 [M, N] tensor in
the epilogue (the decoder's residual stream). ``gemm_accumulate`` adds the
product into an existing fp32 tensor (a gradient sink) with a TMA reduce-add,
so the sink is never read back by the SM. The kernel is this package's own
persistent, warp-specialised tcgen05 kernel (``csrc/gemm_tc.cu``); there is no
per-shape algorithm selection, so a new shape costs one launch.

Every CUDA bf16 product whose dimensions the TMA can address (K and N
multiples of 8, and M when ``a`` is [K, M]) runs on that kernel; CPU tensors
(and other dtypes) use torch, the path the CPU tests compare against.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops._ext import native

__all__ = ["gemm", "gemm_accumulate", "native_ok", "matmul"]


def native_ok(a: torch.Tensor, b: torch.Tensor, a_t: bool, b_t: bool) -> bool:
    """True when ``op(a) · op(b)`` runs on the tcgen05 kernel."""
    if not (a.is_cuda and a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16 and a.dim() == 2 and b.dim() == 2):
        return False
    m = a.shape[1] if a_t else a.shape[0]
    k = a.shape[0] if a_t else a.shape[1]
    n = b.shape[0] if b_t else b.shape[1]
    return k % 8 == 0 and n % 8 == 0 and (not a_t or m % 8 == 0)


def _op(t: torch.Tensor, tr: bool) -> torch.Tensor:
    return t.t() if tr else t


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = True, alpha: float = 1.0,
         out_dtype: torch.dtype | None = None, residual: torch.Tensor | None = None,
         out: torch.Tensor | None = None) -> torch.Tensor:
    """``alpha · op(a) · op(b) [+ residual]``; ``out_dtype`` defaults to the operands' dtype (fp32 is allowed
    for bf16 operands)."""
    m = a.shape[1] if a_t else a.shape[0]
    n = b.shape[0] if b_t else b.shape[1]
    out_dtype = a.dtype if out_dtype is None else out_dtype
    if not native_ok(a, b, a_t, b_t) or (residual is not None and out_dtype != torch.bfloat16):
        acc = torch.float32 if (out_dtype == torch.float32 and a.dtype != torch.float64) else a.dtype
        y = _op(a, a_t).to(acc).matmul(_op(b, b_t).to(acc))
        if alpha != 1.0:
            y = y * alpha
        if residual is not None:
            y = y + residual.to(y.dtype)
        y = y.to(out_dtype)
        if out is not None:
            out.copy_(y)
            return out
        return y
    if out is None:
        out = torch.empty(m, n, dtype=out_dtype, device=a.device)
    native().gemm_tc(out, a.contiguous(), b.contiguous(), a_t, b_t, 0 if out_dtype == torch.bfloat16 else 1,
                     float(alpha), None if residual is None else residual.contiguous())
    return out


def gemm_accumulate(out: torch.Tensor, a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = True,
                    alpha: float = 1.0) -> torch.Tensor:
    """``out += alpha · op(a) · op(b)`` with ``out`` fp32 (contiguous rows)."""
    if not native_ok(a, b, a_t, b_t) or out.dtype != torch.float32:
        out.add_(_op(a, a_t).to(out.dtype).matmul(_op(b, b_t).to(out.dtype)), alpha=alpha)
        return out
    native().gemm_tc(out, a.contiguous(), b.contiguous(), a_t, b_t, 2, float(alpha), None)
    return out


def matmul(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``x @ w`` for ``x`` [..., K] and ``w`` [K, N] (a weight used un-transposed, e.g. ``dy · W``)."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    return gemm(x2, w, b_t=False).reshape(*lead, w.shape[-1])
