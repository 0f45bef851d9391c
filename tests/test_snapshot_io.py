"""Snapshot I/O: HF-layout save/load round trips, the Qwen3.5 multimodal key remap and coverage checks
both ways (the reference's snapshot-loader tests, restated; CPU)."""

from __future__ import annotations

import json

import pytest
import torch

from thundersync_b200.models.io import config_from_snapshot, load_snapshot, save_snapshot


def _qwen3():
    from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM

    torch.manual_seed(0)
    return Qwen3ForCausalLM(PRESETS["tiny"]).to(torch.bfloat16)


def _hybrid():
    from thundersync_b200.models.hybrid import HYBRID_PRESETS, HybridForCausalLM

    torch.manual_seed(0)
    return HybridForCausalLM(HYBRID_PRESETS["hybrid-tiny"]).to(torch.bfloat16)


@pytest.mark.parametrize("make", [_qwen3, _hybrid])
def test_save_load_round_trip_is_exact(make, tmp_path):
    model = make()
    save_snapshot(model, tmp_path)
    kind, cfg = config_from_snapshot(tmp_path)
    assert kind == ("hybrid" if "Hybrid" in type(model).__name__ else "qwen3")
    back = load_snapshot(tmp_path, dtype=torch.bfloat16)
    a, b = model.state_dict(), back.state_dict()
    assert a.keys() == b.keys()
    for k in a:
        assert torch.equal(a[k], b[k]), k
    if getattr(cfg, "tie_word_embeddings", False):
        assert back.lm_head.weight is back.model.embed_tokens.weight


def test_multimodal_snapshot_keys_are_remapped_and_extras_skipped(tmp_path):
    """A Qwen3.5 (vision-language) snapshot stores the text model under model.language_model.* and adds
    visual / mtp weights: the loader maps the former and skips the latter."""
    from safetensors.torch import load_file, save_file

    model = _hybrid()
    save_snapshot(model, tmp_path)
    # clones: the loaded tensors map the file that is rewritten below
    state = {k: v.clone() for k, v in load_file(str(tmp_path / "model.safetensors")).items()}
    remapped = {}
    for k, v in state.items():
        remapped["model.language_model." + k[len("model."):] if k.startswith("model.") else k] = v
    remapped["model.visual.patch_embed.weight"] = torch.zeros(4, 4)
    remapped["mtp.fc.weight"] = torch.zeros(2, 2)
    save_file(remapped, str(tmp_path / "model.safetensors"))
    raw = json.loads((tmp_path / "config.json").read_text())
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "qwen3_5", "text_config": raw}))
    back = load_snapshot(tmp_path)
    for k, v in model.state_dict().items():
        assert torch.equal(v, back.state_dict()[k]), k


def test_coverage_is_checked_both_ways(tmp_path):
    from safetensors.torch import load_file, save_file

    model = _qwen3()
    save_snapshot(model, tmp_path)
    state = {k: v.clone() for k, v in load_file(str(tmp_path / "model.safetensors")).items()}
    missing = dict(state)
    missing.pop(next(k for k in state if "layers.0.mlp.down_proj" in k))
    save_file(missing, str(tmp_path / "model.safetensors"))
    with pytest.raises(RuntimeError, match="missing"):
        load_snapshot(tmp_path)
    extra = dict(state)
    extra["model.layers.0.mlp.extra_proj.weight"] = torch.zeros(2, 2, dtype=torch.bfloat16)
    save_file(extra, str(tmp_path / "model.safetensors"))
    with pytest.raises(RuntimeError, match="match no parameter"):
        load_snapshot(tmp_path)
    bad = dict(state)
    k0 = next(iter(bad))
    bad[k0] = torch.zeros(3, 3, dtype=torch.bfloat16)
    save_file(bad, str(tmp_path / "model.safetensors"))
    with pytest.raises(RuntimeError, match="shape"):
        load_snapshot(tmp_path)


def test_unsupported_family_and_non_directory_are_refused(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "llama"}))
    with pytest.raises(NotImplementedError, match="llama"):
        config_from_snapshot(tmp_path)
    with pytest.raises(ValueError, match="local snapshot directory"):
        load_snapshot(tmp_path / "missing")
