"""Flat-buffer statistic kernels (K15′, K10′): folds, combines, scaled adds.

All operate on the parameter arena's flat layout:

* ``fold_(g1, g2, src, r)``        ``g2 += src``; ``g1 += r·src`` (skipped when r == 0)
* ``axpby_(out, x, y, a, b)``      ``out += a·x + b·y`` (y may be None) -- the
  group-close combine ``(G1 − μ·G2)/σ`` and its binary-reward form
  ``((1−μ)·P − μ·N)/σ``
* ``scale_(x, s)``                 ``x *= s``
* ``reduce_adjoints(out, parts)``  ``out = (out or 0) + Σ parts`` in fp32, fixed
  order, ≤16 parts per launch (the boundary-adjoint reduction of reference
  src/thundersync/engine/boundary_adjoint.py:51-115)

CUDA runs this package's vectorised kernels (16-byte loads, fp32 math,
grid sized to the SM count); CPU runs the same arithmetic in torch.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops._ext import native

MAX_DEGREE = 16


def fold_(g1: torch.Tensor | None, g2: torch.Tensor, src: torch.Tensor, r: float) -> None:
    if g2.is_cuda:
        native().fold_stats(g1, g2, src, float(r))
        return
    g2.add_(src)
    if g1 is not None and r != 0.0:
        g1.add_(src.to(g1.dtype), alpha=float(r))


def axpby_(out: torch.Tensor, x: torch.Tensor, y: torch.Tensor | None, a: float, b: float = 0.0) -> None:
    if out.is_cuda:
        native().axpby(out, x, y, float(a), float(b))
        return
    if y is None:
        out.add_(x.to(out.dtype), alpha=float(a))
    else:
        out.add_(x.to(out.dtype) * float(a) + y.to(out.dtype) * float(b))


def scale_(x: torch.Tensor, s: float) -> None:
    if x.is_cuda:
        native().scale(x, float(s))
    else:
        x.mul_(float(s))


def reduce_adjoints(existing: torch.Tensor | None, parts: list[torch.Tensor]) -> torch.Tensor:
    """``existing + Σ parts`` accumulated in fp32 in list order."""
    if not parts:
        if existing is None:
            raise ValueError("nothing to reduce")
        return existing
    out = existing.float() if existing is not None else torch.zeros_like(parts[0], dtype=torch.float32)
    if existing is not None and existing.dtype == torch.float32:
        out = existing
    if out.is_cuda:
        for i in range(0, len(parts), MAX_DEGREE):
            native().reduce_into(out, [p.contiguous() for p in parts[i : i + MAX_DEGREE]])
        return out
    for p in parts:
        out.add_(p)
    return out
