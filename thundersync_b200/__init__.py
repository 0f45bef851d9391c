"""Blackwell-native streaming-backward GRPO and on-policy distillation.

Public entry points are loaded lazily from their submodules on first access,
so ``import thundersync_b200`` imports neither torch nor the native extension.
The names match the reference package's top-level exports
(reference: src/thundersync/__init__.py:16-29).
"""

from __future__ import annotations

from importlib import import_module
from typing import Any

__version__ = "0.1.0"

_EXPORTS = {
    "ConfigError": "thundersync_b200.config",
    "PolicyModelConfig": "thundersync_b200.config",
    "apply_trainer_determinism": "thundersync_b200.determinism",
    "StreamingRun": "thundersync_b200.engine.streaming",
    "STREAM_ATTENTION_NAME": "thundersync_b200.engine.streaming",
    "register_stream_attention": "thundersync_b200.engine.streaming",
    "RewardLinearBackward": "thundersync_b200.grpo.reward_linear",
    "GrpoTrainerConfig": "thundersync_b200.grpo.config",
    "StreamingTrainerConfig": "thundersync_b200.grpo.config",
    "DataParallelThunderSync": "thundersync_b200.grpo.data_parallel",
    "load_trainer": "thundersync_b200.grpo.runtime",
    "OPDTurnStream": "thundersync_b200.opd.objectives",
    "OPDStream": "thundersync_b200.opd.objectives",
    "Qwen3Config": "thundersync_b200.models.qwen3",
    "Qwen3ForCausalLM": "thundersync_b200.models.qwen3",
    "HybridConfig": "thundersync_b200.models.hybrid",
    "HybridForCausalLM": "thundersync_b200.models.hybrid",
}

__all__ = sorted([*_EXPORTS, "__version__"])


def __getattr__(name: str) -> Any:
    module = _EXPORTS.get(name)
    if module is None:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    value = getattr(import_module(module), name)
    globals()[name] = value
    return value


def __dir__() -> list[str]:
    return sorted({*globals(), *_EXPORTS})
