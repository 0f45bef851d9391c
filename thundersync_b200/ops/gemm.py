"""tcgen05 GEMM (S4): ``out (op)= alpha · op(a) · op(b)`` in bf16 with fp32 accumulation.

``gemm(a, b, a_t=False, b_t=True)`` computes ``a @ b.T`` for an ``nn.Linear``
weight ``b`` [N, K]; ``b_t=False`` takes ``b`` as [K, N]; ``a_t=True`` takes
``a`` as [K, M]. So ``y = x·Wᵀ`` is ``gemm(x, W)``, ``dx = dy·W`` is
``gemm(dy, W, b_t=False)`` and ``dW = dyᵀ·x`` is ``gemm(dy, x, a_t=True,
b_t=False)`` — no transpose copies. ``accumulate_into`` adds the product into
an existing fp32 tensor (a gradient sink). The kernel is this package's own
persistent, warp-specialised tcgen05 kernel (``csrc/gemm_tc.cu``); there is no
per-shape algorithm selection, so a new shape costs one launch.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops._ext import native

__all__ = ["gemm", "gemm_accumulate"]


def gemm(a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = True, alpha: float = 1.0,
         out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    m = a.shape[1] if a_t else a.shape[0]
    n = b.shape[0] if b_t else b.shape[1]
    out = torch.empty(m, n, dtype=out_dtype, device=a.device)
    native().gemm_tc(out, a.contiguous(), b.contiguous(), a_t, b_t, 0 if out_dtype == torch.bfloat16 else 1,
                     float(alpha))
    return out


def gemm_accumulate(out: torch.Tensor, a: torch.Tensor, b: torch.Tensor, *, a_t: bool = False, b_t: bool = True,
                    alpha: float = 1.0) -> torch.Tensor:
    """``out += alpha · op(a) · op(b)`` with ``out`` fp32 and contiguous."""
    native().gemm_tc(out, a.contiguous(), b.contiguous(), a_t, b_t, 2, float(alpha))
    return out
