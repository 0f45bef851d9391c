"""Schedule-independent gradient reduction by logical source (C20).

Readiness decides *when* a source's contribution is computed; it must not
decide the floating-point order in which the logical batch's gradient is
summed. ``CanonicalGradientReducer`` stages each source's fp32 (fp64 for
fp64 inputs) contribution per parameter and folds the sources in a total,
type-tagged canonical order at ``finalize`` (reference:
src/thundersync/engine/objective_ready.py:24-247).

On CUDA the fold runs this package's fixed-order reduction kernel, up to 16
sources per launch into one fp32 accumulator; the per-element order is the
canonical source order, so the result is bitwise identical to sequential
adds in that order and independent of arrival order.
"""

from __future__ import annotations

import time
from typing import Sequence

import torch

from thundersync_b200.ops._ext import native

__all__ = ["CanonicalGradientReducer", "CanonicalSource", "canonical_source_key"]

CanonicalSource = int | str | tuple["CanonicalSource", ...]
_FOLD_DEGREE = 16


def canonical_source_key(source: CanonicalSource) -> tuple:
    """Total, type-stable ordering key: ints < strings < tuples (recursively)."""
    if isinstance(source, bool):
        raise TypeError("boolean values are not valid canonical source IDs")
    if isinstance(source, int):
        return (0, source)
    if isinstance(source, str):
        return (1, source)
    if isinstance(source, tuple):
        return (2, tuple(canonical_source_key(x) for x in source))
    raise TypeError(f"canonical source IDs must contain only ints, strings, and tuples; got {type(source).__name__}")


def _acc_dtype(t: torch.Tensor) -> torch.dtype:
    return torch.float64 if t.dtype == torch.float64 else torch.float32


class CanonicalGradientReducer:
    """Stage per-source parameter gradients; ``finalize`` folds them in canonical source order."""

    def __init__(self, parameter_count: int, *, storage_device: torch.device | str | None = None) -> None:
        if parameter_count < 0:
            raise ValueError("parameter_count must be non-negative")
        self.parameter_count = parameter_count
        self.storage_device = None if storage_device is None else torch.device(storage_device)
        self._by_source: dict[CanonicalSource, list[torch.Tensor | None]] = {}
        self._shapes: list[torch.Size | None] = [None] * parameter_count
        self._devices: list[torch.device | None] = [None] * parameter_count
        self._dtypes: list[torch.dtype | None] = [None] * parameter_count
        self._contributions = 0
        self._bytes = 0
        self._peak_bytes = 0
        self._peak_sources = 0
        self._fold_s = 0.0
        self._materialize_s = 0.0
        self._finalized = False

    @staticmethod
    def _check_source(source: CanonicalSource) -> None:
        canonical_source_key(source)
        try:
            hash(source)
        except TypeError as exc:
            raise TypeError("canonical source ID must be hashable") from exc

    def add(self, source: CanonicalSource, gradients: Sequence[torch.Tensor | None]) -> None:
        if self._finalized:
            raise RuntimeError("cannot add after canonical reduction finalization")
        self._check_source(source)
        if len(gradients) != self.parameter_count:
            raise ValueError(f"received {len(gradients)} gradients for {self.parameter_count} parameters")
        for i, g in enumerate(gradients):
            if g is not None:
                self.add_parameter(source, i, g)

    def add_parameter(self, source: CanonicalSource, parameter_index: int, gradient: torch.Tensor) -> None:
        if self._finalized:
            raise RuntimeError("cannot add after canonical reduction finalization")
        self._check_source(source)
        if not 0 <= parameter_index < self.parameter_count:
            raise IndexError(f"parameter index {parameter_index} is outside [0, {self.parameter_count})")
        if gradient.is_sparse:
            raise NotImplementedError("canonical parameter reduction requires dense gradients")
        shape = self._shapes[parameter_index]
        if shape is None:
            self._shapes[parameter_index] = gradient.shape
            self._devices[parameter_index] = gradient.device
            self._dtypes[parameter_index] = gradient.dtype
        elif shape != gradient.shape:
            raise ValueError(f"parameter {parameter_index}: gradient shape {gradient.shape} does not match "
                             f"established shape {shape}")
        if source not in self._by_source:
            self._by_source[source] = [None] * self.parameter_count
            self._peak_sources = max(self._peak_sources, len(self._by_source))
        bucket = self._by_source[source]
        value = gradient.detach().to(device=self.storage_device or gradient.device, dtype=_acc_dtype(gradient))
        if bucket[parameter_index] is None:
            bucket[parameter_index] = value.clone().contiguous()
            self._bytes += value.numel() * value.element_size()
            self._peak_bytes = max(self._peak_bytes, self._bytes)
        else:
            if bucket[parameter_index].device != value.device:
                raise RuntimeError(f"canonical source {source!r} parameter {parameter_index} received "
                                   "contributions on different devices")
            bucket[parameter_index].add_(value)
        self._contributions += 1

    def _fold(self) -> list[torch.Tensor | None]:
        order = sorted(self._by_source, key=canonical_source_key)
        out: list[torch.Tensor | None] = [None] * self.parameter_count
        for i in range(self.parameter_count):
            parts = [self._by_source[s][i] for s in order if self._by_source[s][i] is not None]
            if not parts:
                continue
            if parts[0].is_cuda and parts[0].dtype == torch.float32 and all(p.device == parts[0].device
                                                                            for p in parts):
                acc = torch.zeros_like(parts[0])
                flat = acc.view(-1)
                for k in range(0, len(parts), _FOLD_DEGREE):
                    native().reduce_into(flat, [p.view(-1) for p in parts[k:k + _FOLD_DEGREE]])
            else:
                acc = parts[0].clone()
                for p in parts[1:]:
                    acc.add_(p)
            out[i] = acc
        return out

    def finalize(self, *, output_devices: Sequence[torch.device | str | None] | None = None,
                 output_dtypes: Sequence[torch.dtype | None] | None = None) -> list[torch.Tensor | None]:
        """Fold in canonical order, cast to each parameter's device/dtype, and consume the ledger."""
        if self._finalized:
            raise RuntimeError("canonical reduction was already finalized")
        if output_devices is not None and len(output_devices) != self.parameter_count:
            raise ValueError("output_devices must align with parameters")
        if output_dtypes is not None and len(output_dtypes) != self.parameter_count:
            raise ValueError("output_dtypes must align with parameters")
        t0 = time.perf_counter()
        result = self._fold()
        self._fold_s += time.perf_counter() - t0
        t0 = time.perf_counter()
        for i, v in enumerate(result):
            if v is None:
                continue
            dev = self._devices[i] if output_devices is None or output_devices[i] is None else torch.device(
                output_devices[i])
            dt = self._dtypes[i] if output_dtypes is None or output_dtypes[i] is None else output_dtypes[i]
            result[i] = v.to(device=dev, dtype=dt)
        self._materialize_s += time.perf_counter() - t0
        self._by_source.clear()
        self._bytes = 0
        self._finalized = True
        return result

    def diagnostics(self) -> dict[str, int | float | bool | str | None]:
        n_tensors = sum(1 for g in self._by_source.values() for t in g if t is not None)
        return {
            "finalized": self._finalized,
            "source_count": len(self._by_source),
            "peak_source_count": self._peak_sources,
            "contribution_count": self._contributions,
            "tensor_count": n_tensors,
            "bytes": self._bytes,
            "peak_bytes": self._peak_bytes,
            "byte_accounting_scope": "resident_canonical_ledger_only",
            "transient_cast_clone_bytes_included": False,
            "canonical_fold_s": self._fold_s,
            "materialization_s": self._materialize_s,
            "canonical_fold_materialization_s": self._fold_s + self._materialize_s,
            "storage_device": None if self.storage_device is None else str(self.storage_device),
        }
