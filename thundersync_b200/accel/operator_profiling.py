"""Named operator ranges for Kineto traces and NVTX timelines.

A range is named ``thundersync::<category>|key=value|...``; the mode is
``off`` (the default: ``operator_range`` returns a shared no-op context, so a
disabled range costs one dict lookup), ``kineto`` (``record_function``),
``nvtx`` (``torch.cuda.nvtx``) or ``both``. The mode comes from
``THUNDERSYNC_OPERATOR_PROFILE_RANGES`` on first use or from
``configure_operator_profiling``; it is process-global so worker threads see
the same setting (reference: src/thundersync/accel/operator_profiling.py:27-161;
the environment variable and range-name format are kept so existing trace
tooling keeps working).
"""

from __future__ import annotations

import os
from contextlib import contextmanager
from typing import Iterator, Mapping

import torch

__all__ = ["PROFILE_RANGES_ENV", "configure_operator_profiling", "device_role", "operator_profiling_enabled",
           "operator_profiling_mode", "operator_range", "range_name"]

PROFILE_RANGES_ENV = "THUNDERSYNC_OPERATOR_PROFILE_RANGES"
_MODES = ("off", "kineto", "nvtx", "both")
_state: dict[str, object] = {"mode": None, "roles": {}}


def _check(mode: str, source: str) -> str:
    m = mode.strip().lower()
    if m not in _MODES:
        raise ValueError(f"{source} must be one of {sorted(_MODES)}, got {mode!r}")
    return m


def _mode() -> str:
    m = _state["mode"]
    if m is None:
        m = _check(os.environ.get(PROFILE_RANGES_ENV, "off"), PROFILE_RANGES_ENV)
        _state["mode"] = m
    return m  # type: ignore[return-value]


def configure_operator_profiling(mode: str, *, device_roles: Mapping[str, str] | None = None) -> None:
    """Set the mode (and optional device → role names, e.g. ``{"cuda:1": "teacher"}``)."""
    _state["mode"] = _check(mode, "operator profiling mode")
    _state["roles"] = {str(torch.device(d)): str(r) for d, r in (device_roles or {}).items()}


def operator_profiling_mode() -> str:
    return _mode()


def operator_profiling_enabled() -> bool:
    return _mode() != "off"


def device_role(device: torch.device | str) -> str:
    key = str(torch.device(device))
    return _state["roles"].get(key, key)  # type: ignore[union-attr]


def range_name(category: str, **fields: object) -> str:
    parts = [f"thundersync::{category}"]
    for k, v in fields.items():
        if v is not None:
            parts.append(f"{k}=" + str(v).replace("|", "/").replace("\n", " "))
    return "|".join(parts)


class _Off:
    def __enter__(self) -> None:
        return None

    def __exit__(self, *exc) -> bool:
        return False


_OFF = _Off()


@contextmanager
def _on(mode: str, name: str) -> Iterator[None]:
    rec = torch.profiler.record_function(name) if mode in ("kineto", "both") else None
    if rec is not None:
        rec.__enter__()
    pushed = False
    try:
        if mode in ("nvtx", "both"):
            torch.cuda.nvtx.range_push(name)
            pushed = True
        yield
    finally:
        if pushed:
            torch.cuda.nvtx.range_pop()
        if rec is not None:
            rec.__exit__(None, None, None)


def operator_range(category: str, *, fields: Mapping[str, object] | None = None, **named: object):
    """A context manager: the shared no-op when off, else a Kineto and/or NVTX range."""
    mode = _mode()
    if mode == "off":
        return _OFF
    merged = dict(fields or {})
    merged.update(named)
    return _on(mode, range_name(category, **merged))
