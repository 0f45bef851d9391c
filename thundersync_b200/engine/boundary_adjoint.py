"""Reduction of consumer adjoints at a shared forest boundary (C19 / K10′).

``parent = existing + Σ consumer adjoints``: a shared segment's backward needs
the sum of its consumers' adjoints, whichever objective produced them
(reference: src/thundersync/engine/boundary_adjoint.py:1-251).

Backends: ``"torch"`` (the default and the numerical reference: sequential
adds in the adjoints' dtype) and ``"native"`` — this package's CUDA kernel,
which reads up to ``NATIVE_MAX_DEGREE`` consumer buffers per launch, adds
them in a fixed order into an fp32 accumulator and rounds once to the
adjoints' dtype (more than 16 consumers run as successive launches into the
same accumulator). ``"triton"`` is accepted as another name for ``"native"``
so existing configurations keep working. The native path is used only for
contiguous CUDA float tensors that do not require grad; anything else takes
the torch path, whose derivative (the upstream gradient copied to each input)
is explicit.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from thundersync_b200.ops._ext import native

__all__ = ["NATIVE_MAX_DEGREE", "SUPPORTED_BACKENDS", "TRITON_MAX_DEGREE", "native_boundary_adjoint_available",
           "reduce_boundary_adjoints"]

NATIVE_MAX_DEGREE = 16
TRITON_MAX_DEGREE = NATIVE_MAX_DEGREE
SUPPORTED_BACKENDS = frozenset(("torch", "native", "triton"))
_DTYPES = (torch.float32, torch.bfloat16)


def native_boundary_adjoint_available() -> bool:
    return torch.cuda.is_available()


def _validate(adjoints, existing) -> list[torch.Tensor]:
    active = [a for a in adjoints if a is not None]
    ref = active[0] if active else existing
    if ref is None:
        return active
    if not ref.is_floating_point():
        raise TypeError(f"boundary adjoints must be floating-point tensors, got {ref.dtype}")
    others = [("adjoint", a) for a in active] + ([("existing", existing)] if existing is not None else [])
    for name, t in others:
        if t.shape != ref.shape:
            raise ValueError(f"{name} shape {tuple(t.shape)} does not match {tuple(ref.shape)}")
        if t.dtype != ref.dtype:
            raise ValueError(f"{name} dtype {t.dtype} does not match {ref.dtype}")
        if t.device != ref.device:
            raise ValueError(f"{name} device {t.device} does not match {ref.device}")
    return active


def _torch_reduce(active, existing):
    ref = active[0] if active else existing
    if ref is None:
        return None
    if any(t.requires_grad for t in active) or (existing is not None and existing.requires_grad):
        out = torch.zeros_like(ref)
        if existing is not None:
            out = out + existing
        for a in active:
            out = out + a
        return out
    out = existing.clone() if existing is not None else torch.zeros_like(ref)
    for a in active:
        out.add_(a)
    return out


def _native_ok(active, existing) -> bool:
    ref = active[0] if active else None
    return bool(ref is not None and ref.is_cuda and ref.dtype in _DTYPES
                and all(t.is_contiguous() and not t.requires_grad for t in active)
                and (existing is None or not existing.requires_grad))


def _native_reduce(active, existing):
    ref = active[0]
    acc = (existing.float().contiguous().clone() if existing is not None
           else torch.zeros(ref.shape, dtype=torch.float32, device=ref.device))
    flat = acc.view(-1)
    for i in range(0, len(active), NATIVE_MAX_DEGREE):
        native().reduce_into(flat, [t.reshape(-1) for t in active[i:i + NATIVE_MAX_DEGREE]])
    return acc if ref.dtype == torch.float32 else acc.to(ref.dtype)


def reduce_boundary_adjoints(adjoints: Sequence[torch.Tensor | None], *, existing: torch.Tensor | None = None,
                             backend: str = "torch") -> torch.Tensor | None:
    """Sum of the non-None ``adjoints`` plus ``existing``; None when all are None. Inputs are not mutated."""
    if backend not in SUPPORTED_BACKENDS:
        raise ValueError(f"boundary adjoint backend must be one of {sorted(SUPPORTED_BACKENDS)}, got {backend!r}")
    active = _validate(adjoints, existing)
    if backend != "torch" and _native_ok(active, existing):
        return _native_reduce(active, existing)
    return _torch_reduce(active, existing)
