"""Hugging Face safetensors snapshots in and out of the native models.

Key names are the Hugging Face ones, so a snapshot written by
``transformers`` loads here and a snapshot written here loads there:

* dense Qwen3: ``model.embed_tokens.weight``, ``model.layers.N.self_attn.*``,
  ``model.layers.N.mlp.*``, ``model.norm.weight``, ``lm_head.weight``;
* the hybrid vision-language snapshot (``model_type: qwen3_5``) ships the
  text stack under ``model.language_model.*`` beside ``model.visual.*`` and
  ``mtp.*``; the text stack is remapped to ``model.*`` and the vision tower
  and multi-token-prediction head are left out. Coverage is checked both
  ways: every parameter must be filled, and every kept checkpoint key must
  land (reference: src/thundersync/policy_model.py:82-179).
"""

from __future__ import annotations

import glob
import json
from pathlib import Path
from typing import Callable

import torch
from torch import nn

__all__ = [
    "HYBRID_EXCLUDED_PREFIXES",
    "HYBRID_SNAPSHOT_MODEL_TYPE",
    "config_from_snapshot",
    "load_state_into",
    "load_snapshot",
    "save_snapshot",
]

HYBRID_EXCLUDED_PREFIXES = ("model.visual.", "mtp.")
HYBRID_SNAPSHOT_MODEL_TYPE = "qwen3_5"
_HYBRID_TEXT_PREFIX = "model.language_model."


def _hybrid_config(raw: dict):
    from thundersync_b200.models.hybrid import HybridConfig

    known = {f for f in HybridConfig.__dataclass_fields__ if f != "extra"}
    kw = {k: v for k, v in raw.items() if k in known}
    rope = raw.get("rope_parameters") or raw.get("rope_scaling") or {}
    if "rope_theta" not in kw and isinstance(rope, dict) and "rope_theta" in rope:
        kw["rope_theta"] = float(rope["rope_theta"])
    if "partial_rotary_factor" not in kw and isinstance(rope, dict) and "partial_rotary_factor" in rope:
        kw["partial_rotary_factor"] = float(rope["partial_rotary_factor"])
    types = raw.get("layer_types")
    if types and "full_attention_interval" not in kw:
        full = [i for i, t in enumerate(types) if t == "full_attention"]
        if full:
            kw["full_attention_interval"] = full[0] + 1
    cfg = HybridConfig(**kw)
    if types and list(types) != cfg.layer_types:
        raise ValueError("hybrid layer_types is not a fixed full-attention interval")
    return cfg


def config_from_snapshot(path: str | Path):
    """(kind, config) of a local snapshot: kind is ``"qwen3"`` or ``"hybrid"``."""
    raw = json.loads((Path(path) / "config.json").read_text())
    mt = raw.get("model_type")
    if mt == HYBRID_SNAPSHOT_MODEL_TYPE:
        return "hybrid", _hybrid_config(raw["text_config"])
    if mt == "qwen3_5_text":
        return "hybrid", _hybrid_config(raw)
    if mt == "qwen3":
        from thundersync_b200.models.qwen3 import Qwen3Config

        return "qwen3", Qwen3Config.from_dict(raw)
    raise NotImplementedError(f"model_type {mt!r} is not a supported policy family (qwen3, qwen3_5)")


def _shards(path: Path) -> list[str]:
    files = sorted(glob.glob(str(path / "model*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no model*.safetensors in {path}")
    return files


def load_state_into(model: nn.Module, path: str | Path, *, remap: Callable[[str], str | None] | None = None,
                    device: torch.device | str | None = None) -> None:
    """Fill every parameter/buffer of ``model`` from a snapshot's shards, checking coverage both ways."""
    from safetensors.torch import load_file

    path = Path(path)
    own = model.state_dict()
    # tied weights appear once in HF checkpoints
    tied = getattr(getattr(model, "config", None), "tie_word_embeddings", False)
    wanted = set(own)
    if tied:
        wanted.discard("lm_head.weight")
    loaded: set[str] = set()
    unexpected: set[str] = set()
    dev = device if device is not None else next(model.parameters()).device
    with torch.no_grad():
        for shard in _shards(path):
            for key, value in load_file(shard, device=str(dev)).items():
                name = remap(key) if remap is not None else key
                if name is None:
                    continue
                if name not in own:
                    unexpected.add(key)
                    continue
                dst = own[name]
                if dst.shape != value.shape:
                    raise RuntimeError(f"checkpoint {key}: shape {tuple(value.shape)} != {tuple(dst.shape)}")
                dst.copy_(value.to(dst.dtype))
                loaded.add(name)
    missing = wanted - loaded
    if missing:
        raise RuntimeError(f"checkpoint coverage: {len(missing)} parameters missing, e.g. {sorted(missing)[:5]}")
    if unexpected:
        raise RuntimeError(
            f"checkpoint coverage: {len(unexpected)} checkpoint keys match no parameter, e.g. {sorted(unexpected)[:5]}")


def _hybrid_remap(key: str) -> str | None:
    if key.startswith(_HYBRID_TEXT_PREFIX):
        return "model." + key[len(_HYBRID_TEXT_PREFIX):]
    if key.startswith(HYBRID_EXCLUDED_PREFIXES):
        return None
    return key


def load_snapshot(path: str | Path, *, device: torch.device | str = "cpu", dtype: torch.dtype = torch.bfloat16):
    """Build the native model of a local snapshot and load its weights."""
    path = Path(path)
    if not path.is_dir():
        raise ValueError(f"the snapshot loader reads a local snapshot directory; {str(path)!r} is not one")
    kind, cfg = config_from_snapshot(path)
    with torch.device("meta"):
        if kind == "hybrid":
            from thundersync_b200.models.hybrid import HybridForCausalLM

            model = HybridForCausalLM(cfg, init=False)
        else:
            from thundersync_b200.models.qwen3 import Qwen3ForCausalLM

            model = Qwen3ForCausalLM(cfg, init=False)
    model = model.to_empty(device=device).to(dtype)
    if cfg.tie_word_embeddings:
        model.lm_head.weight = model.model.embed_tokens.weight
    raw_type = json.loads((path / "config.json").read_text()).get("model_type")
    load_state_into(model, path, remap=_hybrid_remap if raw_type == HYBRID_SNAPSHOT_MODEL_TYPE else None,
                    device=device)
    return model


def save_snapshot(model: nn.Module, path: str | Path, state: dict[str, torch.Tensor] | None = None) -> None:
    """Write ``config.json`` + ``model.safetensors`` (HF key names; tied head written once)."""
    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    cfg = model.config
    state = dict(model.state_dict() if state is None else state)
    if getattr(cfg, "tie_word_embeddings", False):
        state.pop("lm_head.weight", None)
    tensors = {k: v.detach().contiguous().cpu() for k, v in state.items()}
    save_file(tensors, str(path / "model.safetensors"), metadata={"format": "pt"})
    raw = cfg.to_dict()
    if "architectures" not in raw:
        raw["architectures"] = ["Qwen3_5ForCausalLM" if raw.get("model_type") == "qwen3_5_text" else "Qwen3ForCausalLM"]
    raw.setdefault("torch_dtype", "bfloat16")
    (path / "config.json").write_text(json.dumps(raw, indent=2, sort_keys=True))
