"""Loader for the in-tree native extension ``thundersync_b200._C``.

``native()`` returns the module behind a thin proxy that counts how many of
this package's kernels each call launches (``launch_counts``); benchmarks
report that count for their timed region.
"""

from __future__ import annotations

import importlib
import os
import threading
from functools import lru_cache

_LOAD_ERROR: BaseException | None = None

# kernels launched per call of each native entry point
KERNELS_PER_CALL = {
    "rms_norm_fwd": 1, "rms_norm_bwd": 2, "qk_norm_rope_fwd": 1, "qk_norm_rope_bwd": 2,
    "swiglu_fwd": 1, "swiglu_bwd": 1, "embedding_bwd_accumulate": 1, "fold_stats": 1, "axpby": 1,
    "scale": 1, "reduce_into": 1, "lse_gather": 1, "logprob_dlogits": 1,
    "sq_norm": 2, "clip_coef": 1, "adamw_flat": 1,
    "symm_barrier": 1, "ipc_alloc": 0, "ipc_open": 0, "ipc_close": 0, "pinned_slab_alloc": 0, "gemm_tc": 1, "gemm_tc_pair": 0, "gemm_tc_wide": 0, "gemm_tc_epi8": 0, "gemm_tc_direct": 0, "gemm_tc_pdl": 0, "gemm_tc_profile": 0, "gemm_tc_profile_read": 0, "dense_layer_fwd": 10, "dense_layer_bwd": 22, "gemm_tc_cat": 1, "lmhead_lse_tc": 2, "lmhead_dlogits_tc": 1, "tc_selftest": 1, "attn_fwd_tc": 1, "attn_bwd_tc": 3, "attn_fwd_packed": 1, "attn_bwd_packed": 3, "tc_status": 0, "symm_reduce": 1, "symm_reduce_oneshot": 1, "symm_norm_put": 1, "symm_adamw_gather": 1,
    "conv1d_silu_fwd": 1, "conv1d_silu_bwd": 2, "gdn_fwd": 2, "gdn_bwd": 2, "gdn_chunk_fwd": 3, "gdn_chunk_bwd": 3,
}

_lock = threading.Lock()
_calls: dict[str, int] = {}


class _Counted:
    def __init__(self, mod) -> None:
        self._mod = mod
        self.__file__ = mod.__file__

    def __getattr__(self, name: str):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn

        def call(*args, **kwargs):
            with _lock:
                _calls[name] = _calls.get(name, 0) + 1
            return fn(*args, **kwargs)

        call.__name__ = name
        # cached on the instance: later lookups skip __getattr__ entirely
        object.__setattr__(self, name, call)
        return call


@lru_cache(maxsize=1)
def _load():
    global _LOAD_ERROR
    try:
        import torch  # noqa: F401  (the extension links against torch's libraries)

        return _Counted(importlib.import_module("thundersync_b200._C"))
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


def reset_launch_counts() -> None:
    with _lock:
        _calls.clear()


def launch_counts() -> dict[str, int]:
    """Native calls since the last reset, and the kernel launches they made."""
    with _lock:
        calls = dict(_calls)
    kernels = sum(KERNELS_PER_CALL.get(k, 1) * v for k, v in calls.items())
    return {"calls": calls, "kernels": kernels}
