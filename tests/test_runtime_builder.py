"""load_trainer builds (model, optimizer, trainer) from the typed config and steps once (CPU).

Reference behaviour: src/thundersync/grpo/runtime.py:151-319 and
tests/grpo/test_runtime*.py (builder reads only the typed config; LoRA and
sharding options reach the model and optimizer).
"""

from __future__ import annotations

from types import SimpleNamespace

import pytest
import torch

from thundersync_b200.config import ConfigError
from thundersync_b200.grpo.config import GrpoTrainerConfig
from thundersync_b200.grpo.runtime import load_trainer


def _cfg(**kw):
    ns = SimpleNamespace(model_path="random:tiny", learning_rate=1e-3, rebuild_block_tokens=64,
                         deterministic_algorithms=False, **kw)
    return GrpoTrainerConfig.from_namespace(ns)


def test_from_namespace_requires_fields():
    with pytest.raises(ConfigError, match="model_path"):
        GrpoTrainerConfig.from_namespace(SimpleNamespace(learning_rate=1.0, rebuild_block_tokens=1))


@pytest.mark.parametrize("lora", [0, 4])
def test_load_trainer_steps(lora):
    model, opt, trainer = load_trainer(_cfg(lora_rank=lora, source_offload_mode="device_resident"),
                                       torch.device("cpu"))
    trainable = [n for n, p in model.named_parameters() if p.requires_grad]
    if lora:
        assert trainable and all("lora_" in n for n in trainable)
    before = {n: p.detach().clone() for n, p in model.named_parameters() if p.requires_grad}
    trainer.open_group(0, list(range(8)))
    trainer.register_group_trajectories(0, [0, 1])
    for tid, r in ((0, 1.0), (1, 0.0)):
        trainer.append_turn(0, tid, [5 + tid, 6, 7 * (tid + 1)], [True, True, True])
        trainer.close_trajectory(tid, r)
    trainer.close_group(0)
    stats = trainer.step()
    assert stats is not None
    moved = [n for n, p in model.named_parameters() if p.requires_grad and not torch.equal(p, before[n])]
    assert moved


@pytest.mark.parametrize("enabled", [True, False])
def test_load_trainer_applies_determinism_before_the_model_loads(enabled, monkeypatch):
    """The switch is process-wide and must be in force while the policy model is built."""
    import thundersync_b200.policy_model as pm
    from thundersync_b200.determinism import trainer_determinism

    seen = {}

    class Stop(Exception):
        pass

    def fake_load(policy, device):
        seen.update(trainer_determinism())
        raise Stop

    before = trainer_determinism()
    monkeypatch.setattr(pm, "load_policy_model", fake_load)
    try:
        with pytest.raises(Stop):
            load_trainer(GrpoTrainerConfig.from_namespace(SimpleNamespace(
                model_path="random:tiny", learning_rate=1e-3, rebuild_block_tokens=64,
                deterministic_algorithms=enabled)), torch.device("cpu"))
    finally:
        torch.use_deterministic_algorithms(before["deterministic_algorithms"], warn_only=before["warn_only"])
        torch.backends.cudnn.deterministic = before["cudnn_deterministic"]
        torch.backends.cudnn.benchmark = before["cudnn_benchmark"]
    assert seen["deterministic_algorithms"] is enabled and seen["cudnn_deterministic"] is enabled
    assert seen["cudnn_benchmark"] is False and seen["fill_uninitialized_memory"] is False
