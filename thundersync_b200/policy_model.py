"""The policy model a trainer rank trains, its LoRA adapters and its kernels.

Public surface of the reference's ``policy_model`` module
(src/thundersync/policy_model.py:16-28): ``load_policy_model``,
``load_hybrid_causal_lm``, ``apply_lora``, ``lora_target_modules``,
``attach_publication_handle``, ``require_native_bf16``,
``compile_pointwise_modules`` and the target/seed constants.

Differences by design: the model classes are this package's native Qwen3 and
hybrid decoders (Hugging Face key names, native kernels), LoRA is this
package's PEFT-layout adapter (no PEFT dependency), and there is no
``torch.compile`` — the pointwise work already runs as fused CUDA kernels, so
``compile_pointwise_modules`` reports zero modules compiled. A
``model_path`` of the form ``random:<preset>`` builds a random-init model of
a named architecture (used by the benchmark, which has no checkpoints).
"""

from __future__ import annotations

from pathlib import Path

import torch

from thundersync_b200.config import PolicyModelConfig
from thundersync_b200.models.io import HYBRID_EXCLUDED_PREFIXES, HYBRID_SNAPSHOT_MODEL_TYPE, load_snapshot

__all__ = [
    "HYBRID_EXCLUDED_PREFIXES",
    "HYBRID_LORA_TARGETS",
    "HYBRID_SNAPSHOT_MODEL_TYPE",
    "LORA_INIT_SEED",
    "STANDARD_LORA_TARGETS",
    "apply_lora",
    "attach_publication_handle",
    "compile_pointwise_modules",
    "load_hybrid_causal_lm",
    "load_policy_model",
    "lora_target_modules",
    "require_native_bf16",
]

HYBRID_LORA_TARGETS = [
    "q_proj", "k_proj", "v_proj", "o_proj",
    "gate_proj", "up_proj", "down_proj",
    "in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj",
]
STANDARD_LORA_TARGETS = [
    "q_proj", "k_proj", "v_proj", "o_proj",
    "gate_proj", "up_proj", "down_proj",
]
HYBRID_MODEL_TYPES = frozenset({"qwen3_5", "qwen3_5_text"})
LORA_INIT_SEED = 820_042


def compile_pointwise_modules(model: torch.nn.Module) -> int:
    """Accepted for configuration compatibility; returns 0 (nothing is compiled).

    The reference compiles each layer's MLP and norms with Inductor
    (src/thundersync/policy_model.py:38-58). Here those are fused CUDA
    kernels already, and ``torch.compile`` is not on the hot path.
    """
    _decoder_layers(model)
    return 0


def require_native_bf16(device: torch.device) -> None:
    """Refuse a CUDA device without native bf16 arithmetic."""
    device = torch.device(device)
    if device.type != "cuda":
        return
    with torch.cuda.device(device):
        if torch.cuda.is_bf16_supported(including_emulation=False):
            return
        major, minor = torch.cuda.get_device_capability(device)
        name = torch.cuda.get_device_name(device)
    raise RuntimeError(f"the trainer runs in bf16 and {name} (compute capability {major}.{minor}) at {device} "
                       "has no native bf16 support")


def _decoder_layers(model: torch.nn.Module) -> torch.nn.ModuleList:
    layers = getattr(getattr(model, "model", None), "layers", None)
    if not isinstance(layers, torch.nn.ModuleList):
        raise NotImplementedError(f"{type(model).__name__} has no decoder layer stack at model.model.layers; "
                                  "only causal LMs with that layout are supported")
    return layers


def lora_target_modules(model: torch.nn.Module) -> list[str]:
    """Targets ``apply_lora`` wraps: hybrid targets for a hybrid, else the standard seven (all required)."""
    model_type = getattr(getattr(model, "config", None), "model_type", None)
    layers = _decoder_layers(model)
    if model_type in HYBRID_MODEL_TYPES:
        return list(HYBRID_LORA_TARGETS)
    for index, layer in enumerate(layers):
        present = {name.rsplit(".", 1)[-1] for name, m in layer.named_modules() if isinstance(m, torch.nn.Linear)}
        missing = [n for n in STANDARD_LORA_TARGETS if n not in present]
        if missing:
            raise NotImplementedError(f"model_type {model_type!r} is not a supported LoRA family: "
                                      f"decoder layer {index} lacks the linear modules {missing}")
    return list(STANDARD_LORA_TARGETS)


def apply_lora(model: torch.nn.Module, *, rank: int, alpha: int):
    """Inject LoRA adapters in place; return (wrapper, inner model).

    Adapter init is identical across runs and ranks: it draws from the CPU
    generator seeded with ``LORA_INIT_SEED`` inside a forked RNG scope, so the
    caller's RNG state (CPU and CUDA) is unchanged afterwards. Adapters are
    fp32; the frozen base keeps its dtype and ``requires_grad=False``.
    """
    from thundersync_b200.models.lora import LoRAModel, inject_lora

    targets = lora_target_modules(model)
    cuda_devices = sorted({p.device.index for p in model.parameters()
                           if p.device.type == "cuda" and p.device.index is not None})
    model.requires_grad_(False)
    with torch.random.fork_rng(devices=cuda_devices):
        torch.random.default_generator.manual_seed(LORA_INIT_SEED)
        for index in cuda_devices:
            with torch.cuda.device(index):
                torch.cuda.manual_seed(LORA_INIT_SEED)
        inject_lora(model, targets, rank, float(alpha))
    for p in model.parameters():
        if p.requires_grad:
            p.data = p.data.float()
    wrapper = LoRAModel(model, rank=rank, alpha=float(alpha), targets=targets)
    return wrapper, wrapper.base_model.model


def attach_publication_handle(model: torch.nn.Module, peft_model: torch.nn.Module) -> None:
    """Keep the wrapper reachable from the model without registering it as a submodule."""
    object.__setattr__(model, "_thundersync_peft_model", peft_model)


def load_hybrid_causal_lm(snapshot: Path, *, device: torch.device, attn_implementation: str = "native"):
    """Text model + lm_head of a local hybrid vision-language snapshot (keys remapped, coverage checked).
    ``attn_implementation`` is accepted for the reference's signature: attention always runs through this
    package's kernels."""
    if not Path(snapshot).is_dir():
        raise ValueError(f"the hybrid snapshot loader reads a local snapshot directory; {str(snapshot)!r} is not "
                         "one (download the snapshot first)")
    require_native_bf16(device)
    return load_snapshot(snapshot, device=device)


def _random_model(name: str, device: torch.device):
    from thundersync_b200.models.hybrid import HYBRID_PRESETS, HybridForCausalLM
    from thundersync_b200.models.qwen3 import PRESETS, build_qwen3

    torch.manual_seed(0)
    if name in HYBRID_PRESETS:
        with torch.device(device):
            model = HybridForCausalLM(HYBRID_PRESETS[name])
        return model.to(torch.bfloat16)
    if name in PRESETS:
        return build_qwen3(name, device=device, dtype=torch.bfloat16)
    raise ValueError(f"unknown random preset {name!r}")


def load_policy_model(config: PolicyModelConfig, device: torch.device, *, attn_implementation: str = "native"):
    """Policy model of one trainer rank in training mode, with its adapter (if any) attached.
    ``attn_implementation`` is accepted for the reference's signature: attention always runs through this
    package's kernels."""
    device = torch.device(device)
    require_native_bf16(device)
    path = str(config.model_path)
    if path.startswith("random:"):
        model = _random_model(path.split(":", 1)[1], device)
    else:
        model = load_snapshot(Path(path), device=device)
    model.train()
    if config.lora_rank > 0:
        wrapper, model = apply_lora(model, rank=config.lora_rank,
                                    alpha=int(config.lora_alpha or 2 * config.lora_rank))
        model.train()
        attach_publication_handle(model, wrapper)
    else:
        model.requires_grad_(True)
    if config.compile_pointwise_modules:
        compile_pointwise_modules(model)
    return model
