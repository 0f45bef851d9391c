"""Process-wide determinism switch, applied once before the model is built.

``apply_trainer_determinism(True)`` turns on torch's deterministic algorithms
(without NaN-filling fresh allocations) and cuDNN's deterministic selection,
and turns autotuning off. ``False`` turns the first two off and still leaves
autotuning off: packs change length every call, so autotuning would re-run per
shape. The native kernels of this package are deterministic by construction
(fixed reduction orders, no float atomics on gradient paths), so this switch
only governs torch's own ops. Behaviour matches reference
src/thundersync/determinism.py:22-51.
"""

from __future__ import annotations

__all__ = ["apply_trainer_determinism", "trainer_determinism"]


def apply_trainer_determinism(enabled: bool) -> dict[str, bool]:
    if not isinstance(enabled, bool):
        raise TypeError(f"the determinism setting must be a bool, not {enabled!r}")
    import torch
    import torch.utils.deterministic

    torch.use_deterministic_algorithms(enabled)
    torch.utils.deterministic.fill_uninitialized_memory = False
    torch.backends.cudnn.benchmark = False
    torch.backends.cudnn.deterministic = enabled
    return trainer_determinism()


def trainer_determinism() -> dict[str, bool]:
    import torch
    import torch.utils.deterministic

    return {
        "deterministic_algorithms": bool(torch.are_deterministic_algorithms_enabled()),
        "warn_only": bool(torch.is_deterministic_algorithms_warn_only_enabled()),
        "fill_uninitialized_memory": bool(torch.utils.deterministic.fill_uninitialized_memory),
        "cudnn_deterministic": bool(torch.backends.cudnn.deterministic),
        "cudnn_benchmark": bool(torch.backends.cudnn.benchmark),
    }
