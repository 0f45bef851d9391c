"""LoRA adapters in the PEFT module layout, with PEFT-format adapter files.

``LoRALinear`` replaces a target ``nn.Linear`` with the module tree PEFT
builds (``base_layer``, ``lora_A.<adapter>``, ``lora_B.<adapter>``,
``scaling[<adapter>]``), so state-dict keys, the adapter file keys
(``base_model.model.<module path>.lora_A.weight``) and ``adapter_config.json``
are those a PEFT user already has (reference: src/thundersync/policy_model.py:
240-290 wraps the model with ``peft.get_peft_model``; PEFT is not required
here). The forward runs :func:`thundersync_b200.ops.lora.lora_linear`.

Initialisation follows PEFT's ``LoraConfig(init_lora_weights=True)`` for a
``nn.Linear`` target, in the same random-number order, so two runs (and all
ranks) start from identical adapters: for every target in module order, the
A and B ``nn.Linear`` constructors each draw their default init, then A is
re-drawn with ``kaiming_uniform_(a=sqrt(5))`` and B is zeroed. The draws come
from the CPU generator seeded with ``LORA_INIT_SEED``; adapters are fp32.
"""

from __future__ import annotations

import json
import math
from pathlib import Path
from typing import Iterable

import torch
from torch import nn

__all__ = [
    "LoRALinear",
    "LoRAModel",
    "inject_lora",
    "lora_modules",
    "merged_state_dict",
    "save_adapter",
    "load_adapter",
    "adapter_state_dict",
]

ADAPTER = "default"


class LoRALinear(nn.Module):
    """``base_layer(x) + scaling · lora_B(lora_A(x))`` with a frozen base."""

    def __init__(self, base: nn.Linear, rank: int, alpha: float, adapter: str = ADAPTER) -> None:
        super().__init__()
        self.base_layer = base
        self.in_features = base.in_features
        self.out_features = base.out_features
        self.r = {adapter: rank}
        self.lora_alpha = {adapter: alpha}
        self.scaling = {adapter: alpha / rank}
        # constructor draws first (as nn.Linear does), then the LoRA init
        a = nn.Linear(base.in_features, rank, bias=False)
        b = nn.Linear(rank, base.out_features, bias=False)
        nn.init.kaiming_uniform_(a.weight, a=math.sqrt(5))
        nn.init.zeros_(b.weight)
        self.lora_A = nn.ModuleDict({adapter: a})
        self.lora_B = nn.ModuleDict({adapter: b})
        self.active_adapter = adapter
        base.weight.requires_grad_(False)

    @property
    def weight(self) -> torch.Tensor:
        return self.base_layer.weight

    def delta_weight(self, adapter: str | None = None) -> torch.Tensor:
        name = adapter or self.active_adapter
        return (self.lora_B[name].weight.float() @ self.lora_A[name].weight.float()) * self.scaling[name]

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from thundersync_b200.ops.lora import lora_linear

        return lora_linear(x, self, self.active_adapter)


def _matches(name: str, targets: Iterable[str]) -> bool:
    return any(name == t or name.endswith("." + t) for t in targets)


def inject_lora(model: nn.Module, targets: list[str], rank: int, alpha: float) -> list[str]:
    """Replace every ``nn.Linear`` whose name ends in a target; return the replaced names."""
    names = [n for n, m in model.named_modules() if isinstance(m, nn.Linear) and _matches(n, targets)]
    if not names:
        raise ValueError(f"no linear module matches the LoRA targets {targets}")
    for n in names:
        parent_name, _, leaf = n.rpartition(".")
        parent = model.get_submodule(parent_name) if parent_name else model
        base = getattr(parent, leaf)
        lora = LoRALinear(base, rank, alpha)
        dev = base.weight.device
        lora.lora_A.to(device=dev, dtype=torch.float32)
        lora.lora_B.to(device=dev, dtype=torch.float32)
        setattr(parent, leaf, lora)
    return names


def lora_modules(model: nn.Module) -> dict[str, LoRALinear]:
    return {n: m for n, m in model.named_modules() if isinstance(m, LoRALinear)}


def adapter_state_dict(model: nn.Module, adapter: str = ADAPTER) -> dict[str, torch.Tensor]:
    """PEFT adapter-file keys: ``base_model.model.<path>.lora_{A,B}.weight``."""
    out = {}
    for n, m in lora_modules(model).items():
        out[f"base_model.model.{n}.lora_A.weight"] = m.lora_A[adapter].weight.detach()
        out[f"base_model.model.{n}.lora_B.weight"] = m.lora_B[adapter].weight.detach()
    return out


def merged_state_dict(model: nn.Module, dtype: torch.dtype | None = None) -> dict[str, torch.Tensor]:
    """The base model's state dict with every adapter merged (``W + s·B·A``) and LoRA keys dropped."""
    loras = lora_modules(model)
    out = {}
    for key, value in model.state_dict().items():
        if ".lora_A." in key or ".lora_B." in key:
            continue
        mod_name = key.rsplit(".", 2)[0] if ".base_layer." in key else None
        if mod_name is not None and mod_name in loras and key.endswith("base_layer.weight"):
            m = loras[mod_name]
            merged = (value.float() + m.delta_weight()).to(dtype or value.dtype)
            out[f"{mod_name}.weight"] = merged
        else:
            out[key.replace(".base_layer.", ".")] = value if dtype is None else value.to(dtype)
    return out


class LoRAModel(nn.Module):
    """The PEFT-wrapper-shaped handle: ``.base_model.model`` is the adapted model."""

    class _Base(nn.Module):
        def __init__(self, model: nn.Module) -> None:
            super().__init__()
            self.model = model

    def __init__(self, model: nn.Module, *, rank: int, alpha: float, targets: list[str],
                 base_model_name_or_path: str | None = None) -> None:
        super().__init__()
        self.base_model = LoRAModel._Base(model)
        self.peft_config = {
            ADAPTER: {
                "peft_type": "LORA",
                "task_type": "CAUSAL_LM",
                "r": rank,
                "lora_alpha": alpha,
                "lora_dropout": 0.0,
                "bias": "none",
                "target_modules": sorted(targets),
                "fan_in_fan_out": False,
                "init_lora_weights": True,
                "inference_mode": False,
                "base_model_name_or_path": base_model_name_or_path,
                "modules_to_save": None,
            }
        }

    def forward(self, *args, **kwargs):
        return self.base_model.model(*args, **kwargs)

    def save_pretrained(self, directory: str | Path) -> None:
        save_adapter(self.base_model.model, directory, self.peft_config[ADAPTER])

    def merged_state_dict(self, dtype: torch.dtype | None = None) -> dict[str, torch.Tensor]:
        return merged_state_dict(self.base_model.model, dtype)


def save_adapter(model: nn.Module, directory: str | Path, config: dict) -> None:
    """Write ``adapter_model.safetensors`` + ``adapter_config.json``."""
    from safetensors.torch import save_file

    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    tensors = {k: v.contiguous().cpu() for k, v in adapter_state_dict(model).items()}
    save_file(tensors, str(d / "adapter_model.safetensors"), metadata={"format": "pt"})
    cfg = dict(config)
    cfg["inference_mode"] = True
    (d / "adapter_config.json").write_text(json.dumps(cfg, indent=2, sort_keys=True))


def load_adapter(model: nn.Module, directory: str | Path, adapter: str = ADAPTER) -> int:
    """Load a PEFT adapter file into an already-injected model; returns tensors loaded."""
    from safetensors.torch import load_file

    state = load_file(str(Path(directory) / "adapter_model.safetensors"))
    loras = lora_modules(model)
    n = 0
    with torch.no_grad():
        for key, value in state.items():
            if not key.startswith("base_model.model."):
                raise KeyError(f"unexpected adapter key {key}")
            path, kind, _ = key[len("base_model.model."):].rsplit(".", 2)
            mod = loras.get(path)
            if mod is None:
                raise KeyError(f"adapter key {key} has no LoRA module")
            target = (mod.lora_A if kind == "lora_A" else mod.lora_B)[adapter].weight
            target.copy_(value.to(target.dtype))
            n += 1
    expected = 2 * len(loras)
    if n != expected:
        raise RuntimeError(f"adapter file holds {n} tensors, the model has {expected} adapter weights")
    return n
