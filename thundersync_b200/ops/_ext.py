"""Loader for the in-tree native extension ``thundersync_b200._C``."""

from __future__ import annotations

import importlib
import os
from functools import lru_cache

_LOAD_ERROR: BaseException | None = None


@lru_cache(maxsize=1)
def _load():
    global _LOAD_ERROR
    try:
        import torch  # noqa: F401  (the extension links against torch's libraries)

        return importlib.import_module("thundersync_b200._C")
    except BaseException as exc:  # pragma: no cover - depends on build state
        _LOAD_ERROR = exc
        return None


def available() -> bool:
    return _load() is not None


def native():
    """The native module; raises a clear error when it was not built."""
    mod = _load()
    if mod is None:
        raise RuntimeError(
            "thundersync_b200 native extension is not built or failed to load "
            f"({_LOAD_ERROR!r}); run `python setup.py build_ext --inplace` "
            "(the CUDA path has no fallback)"
        )
    return mod


def so_path() -> str | None:
    mod = _load()
    return None if mod is None else os.path.abspath(mod.__file__)
