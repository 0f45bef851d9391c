"""Configuration and public-API contract (the reference's config / API tests, restated).

Every validation rule of the trainer configuration raises ``ConfigError`` naming the field; the
namespace translation requires its three fields, passes bool flags through uncoerced and maps
"none" devices; the package's public names resolve lazily and the determinism switch round-trips.
"""

from __future__ import annotations

import dataclasses
import subprocess
import sys
from pathlib import Path
from types import SimpleNamespace

import pytest

from thundersync_b200.config import ConfigError, PolicyModelConfig
from thundersync_b200.grpo.config import GrpoTrainerConfig, StreamingTrainerConfig

_STREAMING = dict(
    rebuild_block_tokens=4096, rebuild_plain_reserve_gib=0.0, gradient_accumulation_offload_device=None,
    rebuild_checkpoint_storage_device=None, retained_bytes_log_every=0, source_offload_device=None,
    source_offload_mode="blocking", source_offload_window_mib=256, source_offload_hbm_threshold=0.65,
    source_offload_pinned_windows=2, source_reduction_mode="unrestricted_statistics",
    source_reduction_pack_size=1, source_reduction_worker_count=2, source_offload_worker_count=2,
    source_spill_directory=None, statistic_device=None, statistic_dtype="fp32",
)


def _streaming(**kw):
    return StreamingTrainerConfig(**{**_STREAMING, **kw})


def test_defaults_are_valid():
    cfg = _streaming()
    assert cfg.source_pinned_min_slabs == 1 and cfg.direct_when_group_bound is False
    with pytest.raises(dataclasses.FrozenInstanceError):
        cfg.rebuild_block_tokens = 1  # type: ignore[misc]


@pytest.mark.parametrize("kw,field", [
    ({"rebuild_block_tokens": 0}, "rebuild_block_tokens"),
    ({"source_offload_mode": "async"}, "source_offload_mode"),
    ({"source_reduction_mode": "mean"}, "source_reduction_mode"),
    ({"retained_bytes_log_every": -1}, "retained_bytes_log_every"),
    ({"statistic_dtype": "bf16"}, "statistic_dtype"),
    ({"source_pinned_host_fraction": 1.5}, "source_pinned_host_fraction"),
    ({"source_pinned_min_slabs": 0}, "source_pinned_min_slabs"),
    ({"source_pinned_min_slabs": 4, "source_pinned_max_slabs": 2}, "source_pinned_max_slabs"),
    ({"statistic_open_groups": -1}, "statistic_open_groups"),
    ({"statistic_device": "auto"}, "statistic_device"),
    ({"device_statistic_reserve_gib": -1.0}, "device_statistic_reserve_gib"),
    ({"direct_when_group_bound": "yes"}, "direct_when_group_bound"),
    ({"direct_when_group_bound": 1}, "direct_when_group_bound"),
    ({"source_rebuild_block_tokens": -1}, "source_rebuild_block_tokens"),
    ({"source_attention_backend": "flash"}, "source_attention_backend"),
    ({"source_attention_query_chunk": -4}, "source_attention_query_chunk"),
    ({"source_attention_query_chunk": True}, "source_attention_query_chunk"),
    ({"source_attention_kv_bucket": 64}, "source_attention_kv_bucket"),
    ({"source_attention_query_chunk": 64}, "cudnn_graph"),
    ({"release_source_gradients": "on"}, "release_source_gradients"),
    ({"combine_known_reward_sources": 0}, "combine_known_reward_sources"),
    ({"release_source_gradients": True}, "pinned_nonblocking"),
])
def test_streaming_config_rules(kw, field):
    with pytest.raises(ConfigError, match=field):
        _streaming(**kw)


def test_streaming_config_accepts_the_allowed_combinations():
    _streaming(statistic_device="auto", source_offload_mode="device_resident")
    _streaming(source_attention_backend="cudnn_graph", source_attention_query_chunk=64, source_attention_kv_bucket=8)
    _streaming(release_source_gradients=True, source_offload_mode="pinned_nonblocking")


@pytest.mark.parametrize("kw,field", [
    ({"learning_rate": 0.0}, "learning_rate"),
    ({"lora_rank": -1}, "lora_rank"),
    ({"lora_alpha": 0.0, "lora_rank": 8}, "lora_alpha"),
    ({"deterministic_algorithms": "true"}, "deterministic_algorithms"),
    ({"grad_clip": 0.0}, "grad_clip"),
])
def test_policy_config_rules(kw, field):
    base = dict(model_path=Path("m"), disable_fla_causal_conv=False, lora_rank=0, lora_alpha=None, fused_lora=False,
                compile_pointwise_modules=False, learning_rate=1e-5, optimizer_state_sharding=False, grad_clip=1.0,
                deterministic_algorithms=True)
    with pytest.raises(ConfigError, match=field):
        PolicyModelConfig(**{**base, **kw})


@pytest.mark.parametrize("missing", ["model_path", "learning_rate", "rebuild_block_tokens"])
def test_from_namespace_names_each_missing_field(missing):
    ns = {"model_path": "m", "learning_rate": 1e-5, "rebuild_block_tokens": 64}
    ns.pop(missing)
    with pytest.raises(ConfigError, match=missing):
        GrpoTrainerConfig.from_namespace(SimpleNamespace(**ns))


def test_from_namespace_translation():
    cfg = GrpoTrainerConfig.from_namespace(SimpleNamespace(
        model_path="some/model", learning_rate="2e-5", rebuild_block_tokens="128", statistic_device="none",
        max_held_sources=3, prepare_pack_max=5, max_concurrent_groups=6, source_spill_directory="/tmp/spill"))
    assert cfg.policy.model_path == Path("some/model") and cfg.policy.learning_rate == 2e-5
    assert cfg.streaming.rebuild_block_tokens == 128 and cfg.streaming.statistic_device is None
    assert cfg.streaming.source_pinned_min_slabs == 5 and cfg.streaming.source_pinned_max_slabs == 5
    assert cfg.streaming.statistic_open_groups == 6
    assert cfg.streaming.source_spill_directory == Path("/tmp/spill")
    # bool flags are not coerced: a string is refused where a bool is required
    with pytest.raises(ConfigError, match="direct_when_group_bound"):
        GrpoTrainerConfig.from_namespace(SimpleNamespace(model_path="m", learning_rate=1e-5, rebuild_block_tokens=8,
                                                         direct_when_group_bound="off"))


def test_public_names_resolve():
    import thundersync_b200 as ts

    for name in ts.__all__:
        assert getattr(ts, name) is not None, name
    with pytest.raises(AttributeError):
        ts.not_a_name  # noqa: B018


def test_package_import_is_lazy():
    """Importing the package does not import torch (the reference's import contract)."""
    code = "import sys, thundersync_b200; print('torch' in sys.modules)"
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, check=True,
                         cwd=str(Path(__file__).resolve().parents[1]))
    assert out.stdout.strip() == "False"


def test_determinism_switch_round_trip():
    from thundersync_b200.determinism import apply_trainer_determinism, trainer_determinism

    import torch

    before = trainer_determinism()
    try:
        on = apply_trainer_determinism(True)
        assert on["deterministic_algorithms"] and on["cudnn_deterministic"] and not on["cudnn_benchmark"]
        assert not on["fill_uninitialized_memory"]
        off = apply_trainer_determinism(False)
        assert not off["deterministic_algorithms"] and not off["cudnn_benchmark"]
        with pytest.raises(TypeError):
            apply_trainer_determinism("true")  # type: ignore[arg-type]
    finally:
        torch.use_deterministic_algorithms(before["deterministic_algorithms"], warn_only=before["warn_only"])
        torch.backends.cudnn.deterministic = before["cudnn_deterministic"]
        torch.backends.cudnn.benchmark = before["cudnn_benchmark"]
