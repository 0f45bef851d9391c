"""RMSNorm whose backward runs in fp32 while the forward keeps its bytes.

``FP32RMSNormVJP.apply(hidden, weight, eps)`` is this package's RMSNorm op:
the forward rounds exactly as the Hugging Face Qwen3 norm does
(``weight · (x·rsqrt(mean x² + eps)).to(dtype)``) and the backward computes
dx and dw in fp32 with deterministic dw partial sums, on CUDA by this
package's row kernels (reference: src/thundersync/accel/rms_norm.py:7-70,
which calls ATen's ``_fused_rms_norm_backward``).
``use_stable_qwen3_rms_norm`` is kept for configuration compatibility: every
norm of the native models already runs that VJP, so it swaps nothing and
returns how many norms there are. Parameter identity and state-dict keys are
untouched either way.
"""

from __future__ import annotations

import torch

from thundersync_b200.models.qwen3 import RMSNorm
from thundersync_b200.ops.norm import rms_norm

__all__ = ["FP32RMSNormVJP", "StableQwen3RMSNorm", "use_stable_qwen3_rms_norm"]


class FP32RMSNormVJP:
    """``apply(hidden, weight, eps)`` — the function object form of :func:`rms_norm`."""

    @staticmethod
    def apply(hidden: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
        return rms_norm(hidden, weight, float(eps))


class StableQwen3RMSNorm(RMSNorm):
    """The native Qwen3 norm (already an fp32-VJP norm)."""


def use_stable_qwen3_rms_norm(model: torch.nn.Module) -> int:
    return sum(1 for m in model.modules() if isinstance(m, RMSNorm))
