"""Causal-conv routing for hybrid layers.

The reference points each Gated DeltaNet layer's ``causal_conv1d_fn`` at the
FLA Triton convolution (src/thundersync/accel/fla_causal_conv.py:32-79). The
native hybrid model has exactly one convolution, this package's CUDA
conv1d+SiLU kernel with tail chaining, so there is nothing to reroute:
``install_fla_causal_conv`` counts the linear-attention layers that use it
and returns that number (0 for a dense model).
"""

from __future__ import annotations

import torch

__all__ = ["install_fla_causal_conv"]


def install_fla_causal_conv(model: torch.nn.Module) -> int:
    from thundersync_b200.models.hybrid import GatedDeltaNet

    return sum(1 for m in model.modules() if isinstance(m, GatedDeltaNet))
