"""The GRPO trainer builder: typed config → determinism → model → optimizer → DP trainer (C44).

``load_trainer(config, device)`` returns ``(model, optimizer, trainer)``
exactly as the reference's builder does (src/thundersync/grpo/runtime.py:
151-319): every value comes from the typed ``GrpoTrainerConfig``, the
process's determinism switch is applied before the model loads, the model
is the policy of ``config.policy`` (native Qwen3 or hybrid, optional LoRA),
and the trainer is ``DataParallelThunderSync.init_from_env`` with a
``StreamingRun(boundary_cut=True, checkpoint=True, stream_turns=False)``
factory.

B200 choices:

* the optimizer is :class:`~thundersync_b200.parallel.optimizer.FlatAdamW`
  over the flat parameter arena (fp32 master and moments, one fused CUDA
  kernel per step); ``optimizer_state_sharding`` gives each rank a contiguous
  arena shard whose update is the fused reduce-scatter → AdamW → parameter
  all-gather over NVLink;
* ``source_attention_backend`` (``auto``/``cudnn``/``cudnn_graph`` in the
  reference) is accepted and recorded, but every backend name runs this
  package's tcgen05 attention: there is one attention implementation;
* statistics: ``statistic_device="auto"`` with device-resident sources
  places as many open groups' fp32 pairs on the device as
  :func:`device_statistic_slots` finds room for, the rest on the host.
"""

from __future__ import annotations

import logging
import os
from typing import Any

import torch

from thundersync_b200.config import ConfigError
from thundersync_b200.determinism import apply_trainer_determinism
from thundersync_b200.grpo.config import GrpoTrainerConfig, StreamingTrainerConfig
from thundersync_b200.grpo.device_statistics import device_statistic_slots

log = logging.getLogger(__name__)

__all__ = ["load_trainer", "pinned_source_arena", "statistic_placement"]

# AdamW keeps two fp32 moments per trainable element plus the fp32 master.
_OPTIMIZER_STATE_TENSORS = 3


def statistic_placement(config: StreamingTrainerConfig, model: torch.nn.Module, *, owned_numel: int,
                        optimizer_state_tensors: int = _OPTIMIZER_STATE_TENSORS) -> tuple[str | None, int | None]:
    """(statistic device, device statistic slots) for this rank."""
    if config.statistic_device is None:
        return None, None
    if config.source_offload_mode != "device_resident":
        return config.statistic_device, None
    if config.statistic_open_groups < 1:
        raise ConfigError("device statistic homes are sized by the rank's open groups, which the entry point did "
                          "not set")
    if config.statistic_device != "auto":
        return config.statistic_device, config.statistic_open_groups
    params = list(model.parameters())
    trainable = [p for p in params if p.requires_grad]
    device = trainable[0].device
    if device.type != "cuda":
        raise ConfigError("statistic_device auto needs a CUDA parameter device")

    def nbytes(ts):
        return sum(t.numel() * t.element_size() for t in ts)

    src = nbytes(trainable)
    stat = src if config.statistic_dtype == "source" else sum(p.numel() * 4 for p in trainable)
    slots = device_statistic_slots(
        device_total_bytes=int(torch.cuda.get_device_properties(device).total_memory),
        parameter_bytes=nbytes(params) + nbytes(list(model.buffers())), gradient_bytes=4 * sum(
            p.numel() for p in trainable),
        optimizer_state_bytes=optimizer_state_tensors * 4 * owned_numel, source_bytes=src,
        device_held_sources=config.source_pinned_min_slabs, statistic_pair_bytes=2 * stat,
        reserve_bytes=int(config.device_statistic_reserve_gib * (1 << 30)), open_groups=config.statistic_open_groups)
    return "cuda", slots


def pinned_source_arena(config: StreamingTrainerConfig, model: torch.nn.Module):
    """This rank's pinned source slabs (pinned_nonblocking sources with a host fraction), else None."""
    if config.source_offload_mode != "pinned_nonblocking" or config.source_pinned_host_fraction <= 0.0:
        return None
    from thundersync_b200.grpo.pinned_arena import PinnedSourceArena, host_ranks_from_env

    trainable = [p for p in model.parameters() if p.requires_grad]
    src = sum(p.numel() * p.element_size() for p in trainable)
    reserved = 0
    if config.statistic_device is None:  # host statistics share the host budget
        reserved = config.statistic_open_groups * 2 * sum(p.numel() * 4 for p in trainable)
    return PinnedSourceArena.for_host(src, host_ranks=host_ranks_from_env(),
                                      host_fraction=config.source_pinned_host_fraction, reserved_bytes=reserved,
                                      min_slabs=config.source_pinned_min_slabs,
                                      max_slabs=config.source_pinned_max_slabs)


def load_trainer(config: GrpoTrainerConfig, device: torch.device) -> tuple[torch.nn.Module, Any, Any]:
    """Build the policy model, its optimizer and the data-parallel streaming trainer."""
    from thundersync_b200.engine.streaming import StreamingRun, arena_for
    from thundersync_b200.grpo.data_parallel import DataParallelThunderSync, _init_process_group
    from thundersync_b200.parallel.optimizer import FlatAdamW
    from thundersync_b200.policy_model import load_policy_model

    device = torch.device(device)
    apply_trainer_determinism(config.policy.deterministic_algorithms)
    if config.streaming.source_attention_backend != "auto":
        log.info("source_attention_backend=%s runs the native tcgen05 attention",
                 config.streaming.source_attention_backend)
    model = load_policy_model(config.policy, device)
    if config.policy.fused_lora:
        from thundersync_b200.accel.fused_lora import fuse_merged_lora_forward

        wrapper = getattr(model, "_thundersync_peft_model", None)
        if wrapper is not None:
            fuse_merged_lora_forward(wrapper)
    arena = arena_for(model)
    if arena is None:
        raise ConfigError("the trainable parameters must share one device and dtype")
    opt_kw = dict(lr=config.policy.learning_rate, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.0, maximize=True)
    if config.policy.optimizer_state_sharding:
        if "WORLD_SIZE" in os.environ:
            _init_process_group(device, 600.0)
        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("optimizer state sharding requires an initialized process group")
        optimizer = FlatAdamW.sharded(arena, **opt_kw)
    else:
        optimizer = FlatAdamW(arena, **opt_kw)
    stat_dev, slots = statistic_placement(config.streaming, model, owned_numel=optimizer.hi - optimizer.lo)
    st = config.streaming

    def run_factory(owned_model):
        return StreamingRun(
            owned_model, boundary_cut=True, checkpoint=True, stream_turns=False,
            rebuild_block_tokens=st.source_rebuild_block_tokens or st.rebuild_block_tokens,
            rebuild_plain_reserve_bytes=None if st.rebuild_plain_reserve_gib <= 0 else int(
                st.rebuild_plain_reserve_gib * (1 << 30)),
            rebuild_checkpoint_storage_device=st.rebuild_checkpoint_storage_device,
            parameter_adjoint_storage_device=st.gradient_accumulation_offload_device)

    if stat_dev == "cuda":
        stat_dev = device
    trainer = DataParallelThunderSync.init_from_env(
        model, optimizer, source_pinned_arena=pinned_source_arena(st, model), run_factory=run_factory,
        eps=config.grpo_epsilon, grad_clip=config.policy.grad_clip, source_offload_device=st.source_offload_device,
        source_offload_mode=st.source_offload_mode, source_offload_window_bytes=st.source_offload_window_mib << 20,
        source_offload_hbm_threshold=st.source_offload_hbm_threshold, source_reduction_mode=st.source_reduction_mode,
        source_reduction_pack_size=st.source_reduction_pack_size,
        source_reduction_worker_count=st.source_reduction_worker_count,
        source_offload_worker_count=st.source_offload_worker_count,
        source_offload_pinned_windows=st.source_offload_pinned_windows,
        source_spill_directory=st.source_spill_directory, statistic_device=stat_dev, device_statistic_slots=slots,
        statistic_keep_source_dtype=st.statistic_dtype == "source",
        retained_bytes_log_every=st.retained_bytes_log_every, direct_when_group_bound=st.direct_when_group_bound,
        source_release_during_backward=st.release_source_gradients,
        combine_known_reward_sources=st.combine_known_reward_sources)
    return model, optimizer, trainer
