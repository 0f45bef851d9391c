"""Per-device kernel trials: does kernel K run on this device, dtype and shape class?

A trial is a caller-supplied tiny forward+backward; it runs at most once per
(kernel, device index, dtype, shape key), with the device synchronised so an
asynchronous launch failure is attributed to the trial, and the outcome is
recorded with the device's name and compute capability. There are no
architecture lists: what runs is what a trial saw run (reference:
src/thundersync/accel/capability.py:41-129).

This framework's own ops do not consult trials on their hot path — each op
has exactly one CUDA implementation and raises if it cannot run — so trials
serve diagnostics and callers that want to gate optional work.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass
from typing import Callable

import torch

__all__ = ["device_identity", "kernel_runs", "kernel_probe_records", "reset_kernel_probes"]


@dataclass(frozen=True)
class _Outcome:
    runs: bool
    error: str | None


_LOCK = threading.Lock()
_OUTCOMES: dict[tuple[str, int, str, int], _Outcome] = {}


def device_identity(device: torch.device | int | None = None) -> dict[str, object]:
    """Index, name, compute capability and memory (MiB) of a CUDA device; ``{}`` without CUDA."""
    if not torch.cuda.is_available():
        return {}
    if isinstance(device, int):
        index = device
    elif device is not None and torch.device(device).index is not None:
        index = torch.device(device).index
    else:
        index = torch.cuda.current_device()
    p = torch.cuda.get_device_properties(index)
    return {"index": index, "name": p.name, "compute_capability": f"{p.major}.{p.minor}",
            "total_memory_mib": p.total_memory // (1 << 20)}


def _run_trial(trial, device, dtype, shape_key) -> _Outcome:
    try:
        with torch.cuda.device(device), torch.enable_grad():
            trial(device, dtype, shape_key)
            torch.cuda.synchronize(device)
    except Exception as exc:  # noqa: BLE001 - any failure means "does not run here"
        return _Outcome(False, f"{type(exc).__name__}: {str(exc)[:300]}")
    return _Outcome(True, None)


def kernel_runs(kernel: str, like: torch.Tensor, shape_key: int,
                trial: Callable[[torch.device, torch.dtype, int], None]) -> bool:
    """Whether ``trial(device, dtype, shape_key)`` completes on ``like``'s device and dtype."""
    if not like.is_cuda:
        return False
    key = (kernel, like.device.index, str(like.dtype), int(shape_key))
    got = _OUTCOMES.get(key)
    if got is None:
        with _LOCK:
            got = _OUTCOMES.get(key)
            if got is None:
                got = _run_trial(trial, like.device, like.dtype, shape_key)
                _OUTCOMES[key] = got
    return got.runs


def kernel_probe_records() -> list[dict[str, object]]:
    """Every trial this process ran, with the identity of the device it ran on."""
    ids: dict[int, dict[str, object]] = {}
    out = []
    for (kernel, index, dtype, shape_key), o in sorted(_OUTCOMES.items()):
        if index not in ids:
            ids[index] = device_identity(index)
        out.append({"kernel": kernel, "device": ids[index], "dtype": dtype, "shape_key": shape_key,
                    "runs": o.runs, "error": o.error})
    return out


def reset_kernel_probes() -> None:
    with _LOCK:
        _OUTCOMES.clear()
