"""Typed GRPO trainer configuration (C03).

Field names, defaults and validation rules match the reference's
``StreamingTrainerConfig``/``GrpoTrainerConfig`` (src/thundersync/grpo/config.py:60-296)
so that entry-point arguments carry over unchanged. Options that select
between the reference's attention backends are accepted and validated; this
framework has one native attention path, so they do not change execution.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Any

from thundersync_b200.config import ConfigError, PolicyModelConfig

__all__ = [
    "DEFAULT_GRPO_EPSILON",
    "DEFAULT_PINNED_HOST_FRACTION",
    "DEFAULT_SOURCE_OFFLOAD_HBM_THRESHOLD",
    "GrpoTrainerConfig",
    "StreamingTrainerConfig",
    "SOURCE_OFFLOAD_MODES",
    "SOURCE_REDUCTION_MODES",
    "STATISTIC_DTYPES",
]

DEFAULT_GRPO_EPSILON = 1e-6
DEFAULT_PINNED_HOST_FRACTION = 0.8
DEFAULT_SOURCE_OFFLOAD_HBM_THRESHOLD = 0.65
SOURCE_OFFLOAD_MODES = ("blocking", "pinned_nonblocking", "pinned_streaming", "device_resident")
SOURCE_REDUCTION_MODES = ("unrestricted_statistics",)
STATISTIC_DTYPES = ("fp32", "source")


def _optional_path(value: Any) -> Path | None:
    return None if value is None else Path(value)


def _is_bool(v: Any) -> bool:
    return isinstance(v, bool)


@dataclass(frozen=True, slots=True)
class StreamingTrainerConfig:
    """Close rebuild, source/statistic residency and the direct path."""

    rebuild_block_tokens: int
    rebuild_plain_reserve_gib: float
    gradient_accumulation_offload_device: str | None
    rebuild_checkpoint_storage_device: str | None
    retained_bytes_log_every: int
    source_offload_device: str | None
    source_offload_mode: str
    source_offload_window_mib: int
    source_offload_hbm_threshold: float
    source_offload_pinned_windows: int
    source_reduction_mode: str
    source_reduction_pack_size: int
    source_reduction_worker_count: int
    source_offload_worker_count: int
    source_spill_directory: Path | None
    statistic_device: str | None
    statistic_dtype: str
    source_pinned_host_fraction: float = DEFAULT_PINNED_HOST_FRACTION
    source_pinned_min_slabs: int = 1
    source_pinned_max_slabs: int | None = None
    statistic_open_groups: int = 0
    device_statistic_reserve_gib: float = 0.0
    direct_when_group_bound: bool = False
    source_rebuild_block_tokens: int = 0
    source_attention_backend: str = "auto"
    source_attention_query_chunk: int = 0
    source_attention_kv_bucket: int = 0
    release_source_gradients: bool = False
    combine_known_reward_sources: bool = False

    def __post_init__(self) -> None:
        if self.rebuild_block_tokens < 1:
            raise ConfigError("rebuild_block_tokens: expected a positive token count")
        if self.source_offload_mode not in SOURCE_OFFLOAD_MODES:
            raise ConfigError(f"source_offload_mode: expected one of {SOURCE_OFFLOAD_MODES}, got {self.source_offload_mode!r}")
        if self.source_reduction_mode not in SOURCE_REDUCTION_MODES:
            raise ConfigError(f"source_reduction_mode: expected one of {SOURCE_REDUCTION_MODES}, got {self.source_reduction_mode!r}")
        if self.retained_bytes_log_every < 0:
            raise ConfigError("retained_bytes_log_every: expected 0 (off) or a positive interval")
        if self.statistic_dtype not in STATISTIC_DTYPES:
            raise ConfigError(f"statistic_dtype: expected one of {STATISTIC_DTYPES}, got {self.statistic_dtype!r}")
        if not 0.0 <= self.source_pinned_host_fraction <= 1.0:
            raise ConfigError("source_pinned_host_fraction: expected a fraction between 0 and 1")
        if self.source_pinned_min_slabs < 1:
            raise ConfigError("source_pinned_min_slabs: expected at least one slab")
        if self.source_pinned_max_slabs is not None and self.source_pinned_max_slabs < self.source_pinned_min_slabs:
            raise ConfigError("source_pinned_max_slabs: expected a cap of at least source_pinned_min_slabs")
        if self.statistic_open_groups < 0:
            raise ConfigError("statistic_open_groups: expected 0 (unset) or a positive group count")
        if self.statistic_device == "auto" and self.source_offload_mode != "device_resident":
            raise ConfigError("statistic_device='auto' sizes device homes for device_resident sources; set source_offload_mode='device_resident'")
        if self.device_statistic_reserve_gib < 0.0:
            raise ConfigError("device_statistic_reserve_gib: expected a non-negative reserve in GiB")
        if not _is_bool(self.direct_when_group_bound):
            raise ConfigError("direct_when_group_bound: expected a bool")
        if self.source_rebuild_block_tokens < 0:
            raise ConfigError("source_rebuild_block_tokens: expected 0 (inherit) or a positive token count")
        if self.source_attention_backend not in ("auto", "cudnn", "cudnn_graph"):
            raise ConfigError(f"source_attention_backend: expected 'auto', 'cudnn' or 'cudnn_graph', got {self.source_attention_backend!r}")
        for name in ("source_attention_query_chunk", "source_attention_kv_bucket"):
            v = getattr(self, name)
            if not isinstance(v, int) or isinstance(v, bool) or v < 0:
                raise ConfigError(f"{name}: expected a non-negative int")
        if self.source_attention_kv_bucket and not self.source_attention_query_chunk:
            raise ConfigError("source_attention_kv_bucket only applies with a source_attention_query_chunk")
        if (self.source_attention_query_chunk or self.source_attention_kv_bucket) and (
            self.source_attention_backend != "cudnn_graph"
        ):
            raise ConfigError("source_attention_query_chunk / source_attention_kv_bucket apply to the cudnn_graph backend only")
        for name in ("release_source_gradients", "combine_known_reward_sources"):
            if not _is_bool(getattr(self, name)):
                raise ConfigError(f"{name}: expected a bool")
        if self.release_source_gradients and self.source_offload_mode != "pinned_nonblocking":
            raise ConfigError("release_source_gradients applies to pinned_nonblocking sources only")


@dataclass(frozen=True, slots=True)
class GrpoTrainerConfig:
    """Everything the GRPO trainer builder reads about one run."""

    policy: PolicyModelConfig
    streaming: StreamingTrainerConfig
    grpo_epsilon: float = DEFAULT_GRPO_EPSILON

    @classmethod
    def from_namespace(cls, args: Any) -> "GrpoTrainerConfig":
        """Translate an entry point's parsed arguments.

        ``model_path``, ``learning_rate`` and ``rebuild_block_tokens`` are
        required (a missing one raises ``ConfigError`` naming it); every other
        value falls back to the builder's default. Bool flags pass through
        uncoerced so a string such as ``"off"`` is refused.
        """

        def required(name: str) -> Any:
            if not hasattr(args, name):
                raise ConfigError(f"the trainer configuration needs {name!r}; the parsed arguments do not provide it")
            return getattr(args, name)

        def probe(name: str, default: Any) -> Any:
            return getattr(args, name, default)

        def device(name: str) -> str | None:
            value = probe(name, None)
            return None if value == "none" else value

        held = int(probe("max_held_sources", 0) or 0)
        pack = int(probe("prepare_pack_max", 0) or 0)
        policy = PolicyModelConfig(
            model_path=Path(required("model_path")),
            disable_fla_causal_conv=bool(probe("disable_fla_causal_conv", False)),
            lora_rank=int(probe("lora_rank", 0) or 0),
            lora_alpha=probe("lora_alpha", None),
            fused_lora=bool(probe("fused_lora", False)),
            compile_pointwise_modules=bool(probe("compile_pointwise_modules", False)),
            learning_rate=float(required("learning_rate")),
            optimizer_state_sharding=bool(probe("optimizer_state_sharding", False)),
            grad_clip=float(probe("grad_clip", 1.0)),
            deterministic_algorithms=probe("deterministic_algorithms", True),
        )
        streaming = StreamingTrainerConfig(
            rebuild_block_tokens=int(required("rebuild_block_tokens")),
            rebuild_plain_reserve_gib=float(probe("rebuild_plain_reserve_gib", 0.0)),
            rebuild_checkpoint_storage_device=device("rebuild_checkpoint_storage_device"),
            gradient_accumulation_offload_device=device("gradient_accumulation_offload_device"),
            source_offload_device=probe("source_offload_device", None),
            source_offload_mode=str(probe("source_offload_mode", "blocking")),
            source_offload_window_mib=int(probe("source_offload_window_mib", 256)),
            source_offload_hbm_threshold=float(
                probe("source_offload_hbm_threshold", DEFAULT_SOURCE_OFFLOAD_HBM_THRESHOLD)
            ),
            source_offload_pinned_windows=int(probe("source_offload_pinned_windows", 2)),
            source_reduction_mode=str(probe("source_reduction_mode", "unrestricted_statistics")),
            source_reduction_pack_size=int(probe("source_reduction_pack_size", 1)),
            source_reduction_worker_count=int(probe("source_reduction_worker_count", 2)),
            source_offload_worker_count=int(probe("source_offload_worker_count", 2)),
            source_spill_directory=_optional_path(probe("source_spill_directory", None)),
            statistic_device=device("statistic_device"),
            statistic_dtype=str(probe("statistic_dtype", "fp32")),
            retained_bytes_log_every=int(probe("retained_bytes_log_every", 0)),
            source_pinned_host_fraction=float(probe("pinned_host_fraction", DEFAULT_PINNED_HOST_FRACTION)),
            source_pinned_min_slabs=max(1, held, pack),
            source_pinned_max_slabs=(max(held, pack) if held > 0 else None),
            statistic_open_groups=int(
                probe("statistic_open_groups", 0) or probe("max_concurrent_groups", 0) or 0
            ),
            device_statistic_reserve_gib=float(probe("device_statistic_reserve_gib", 0.0) or 0.0),
            direct_when_group_bound=probe("direct_when_group_bound", False),
            source_rebuild_block_tokens=int(probe("source_rebuild_block_tokens", 0)),
            source_attention_backend=str(probe("source_attention_backend", "auto")),
            source_attention_query_chunk=int(probe("source_attention_query_chunk", 0)),
            source_attention_kv_bucket=int(probe("source_attention_kv_bucket", 0)),
            release_source_gradients=probe("release_source_gradients", False),
            combine_known_reward_sources=probe("combine_known_reward_sources", False),
        )
        return cls(policy=policy, streaming=streaming, grpo_epsilon=float(probe("grpo_epsilon", DEFAULT_GRPO_EPSILON)))
