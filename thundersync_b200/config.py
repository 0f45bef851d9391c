"""Trainer configuration shared by every objective and the error it raises.

Field names follow the reference's ``PolicyModelConfig`` so that a caller's
configuration carries over unchanged (reference: src/thundersync/config.py:12-52).
Frozen, slotted, no defaults: each entry point supplies its own.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

__all__ = ["ConfigError", "PolicyModelConfig"]


class ConfigError(ValueError):
    """Raised for a configuration a trainer refuses to accept."""


@dataclass(frozen=True, slots=True)
class PolicyModelConfig:
    """The policy model one trainer rank builds, and its optimizer settings.

    ``model_path`` is a local safetensors snapshot directory, or the special
    form ``random:<arch>`` (for example ``random:qwen3-1.7b``) which builds a
    random-init model of a named architecture with no files at all.
    ``disable_fla_causal_conv`` and ``compile_pointwise_modules`` are accepted
    for configuration compatibility; this framework has exactly one native
    conv1d and one set of fused pointwise kernels, so both are no-ops.
    """

    model_path: Path
    disable_fla_causal_conv: bool
    lora_rank: int
    lora_alpha: int | None
    fused_lora: bool
    compile_pointwise_modules: bool
    learning_rate: float
    optimizer_state_sharding: bool
    grad_clip: float
    deterministic_algorithms: bool

    def __post_init__(self) -> None:
        if not (self.learning_rate > 0.0):
            raise ConfigError("learning_rate: expected a positive value")
        if self.lora_rank < 0:
            raise ConfigError("lora_rank: expected 0 (full fine-tune) or a positive rank")
        if self.lora_alpha is not None and self.lora_alpha <= 0:
            raise ConfigError("lora_alpha: expected a positive value or None")
        if not isinstance(self.deterministic_algorithms, bool):
            raise ConfigError("deterministic_algorithms: expected a bool")
        if not (self.grad_clip > 0.0):
            raise ConfigError("grad_clip: expected a positive max norm")
