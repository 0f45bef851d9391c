"""Native Qwen3 dense decoder with Hugging Face-compatible parameter names.

The module tree mirrors ``transformers``' Qwen3 layout (``model.embed_tokens``,
``model.layers.N.self_attn.{q,k,v,o}_proj``, ``q_norm``/``k_norm``,
``mlp.{gate,up,down}_proj``, ``input_layernorm``, ``post_attention_layernorm``,
``model.norm``, ``lm_head``) so safetensors snapshots and PEFT adapters load
with identical keys (reference: src/thundersync/policy_model.py:322-377 loads
the HF class; this framework owns the layer instead so it can fuse
norm/QK-norm/RoPE/attention/LM-head into its own sm_100a kernels).

Execution never goes through an HF forward: ``thundersync_b200.engine.layers``
reads these parameters and runs the native ops. ``forward`` here is the plain
full-causal forward used by tests and the oracle.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field, replace
from typing import Any

import torch
from torch import nn

__all__ = [
    "Qwen3Config",
    "Qwen3ForCausalLM",
    "Qwen3Model",
    "Qwen3DecoderLayer",
    "RMSNorm",
    "PRESETS",
]


@dataclass(frozen=True)
class Qwen3Config:
    vocab_size: int = 151936
    hidden_size: int = 2048
    intermediate_size: int = 6144
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    tie_word_embeddings: bool = True
    max_position_embeddings: int = 40960
    initializer_range: float = 0.02
    qk_norm: bool = True
    model_type: str = "qwen3"
    extra: dict = field(default_factory=dict, compare=False, hash=False)

    def to_dict(self) -> dict[str, Any]:
        out = asdict(self)
        out.pop("extra")
        out.update(self.extra)
        out["architectures"] = ["Qwen3ForCausalLM"]
        return out

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> "Qwen3Config":
        known = {f for f in cls.__dataclass_fields__ if f != "extra"}
        kwargs = {k: v for k, v in data.items() if k in known}
        if "rope_theta" not in kwargs:
            rope = data.get("rope_parameters") or data.get("rope_scaling") or {}
            if isinstance(rope, dict) and "rope_theta" in rope:
                kwargs["rope_theta"] = float(rope["rope_theta"])
        if kwargs.get("head_dim") is None:
            kwargs["head_dim"] = data["hidden_size"] // data["num_attention_heads"]
        return cls(**kwargs)

    def with_(self, **changes: Any) -> "Qwen3Config":
        return replace(self, **changes)

    @property
    def n_params(self) -> int:
        d, f, v = self.hidden_size, self.intermediate_size, self.vocab_size
        hq, hk, hd = self.num_attention_heads, self.num_key_value_heads, self.head_dim
        per_layer = d * hq * hd + 2 * d * hk * hd + hq * hd * d + 3 * d * f + 2 * d
        per_layer += 2 * hd if self.qk_norm else 0
        head = 0 if self.tie_word_embeddings else v * d
        return v * d + self.num_hidden_layers * per_layer + d + head


# Architectures named by the benchmark configurations. Dimensions are the
# public Qwen3 model cards' (vocab 151936, RoPE theta 1e6, RMSNorm eps 1e-6).
PRESETS: dict[str, Qwen3Config] = {
    "qwen3-1.7b": Qwen3Config(
        hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
        num_attention_heads=16, num_key_value_heads=8, head_dim=128, tie_word_embeddings=True,
    ),
    "qwen3-4b": Qwen3Config(
        hidden_size=2560, intermediate_size=9728, num_hidden_layers=36,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, tie_word_embeddings=True,
    ),
    "qwen3-8b": Qwen3Config(
        hidden_size=4096, intermediate_size=12288, num_hidden_layers=36,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, tie_word_embeddings=False,
    ),
    # The CPU correctness configuration: 2 layers, hidden 64, 4q/2kv heads of 16.
    "tiny": Qwen3Config(
        vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=16, tie_word_embeddings=True,
        max_position_embeddings=4096,
    ),
}


class RMSNorm(nn.Module):
    """Weight-only RMSNorm; the math lives in ``thundersync_b200.ops.norm``."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from thundersync_b200.ops.norm import rms_norm

        return rms_norm(x, self.weight, self.variance_epsilon)


class Qwen3Attention(nn.Module):
    def __init__(self, cfg: Qwen3Config, layer_idx: int) -> None:
        super().__init__()
        d, hd = cfg.hidden_size, cfg.head_dim
        self.layer_idx = layer_idx
        self.head_dim = hd
        self.num_heads = cfg.num_attention_heads
        self.num_key_value_heads = cfg.num_key_value_heads
        self.q_proj = nn.Linear(d, cfg.num_attention_heads * hd, bias=False)
        self.k_proj = nn.Linear(d, cfg.num_key_value_heads * hd, bias=False)
        self.v_proj = nn.Linear(d, cfg.num_key_value_heads * hd, bias=False)
        self.o_proj = nn.Linear(cfg.num_attention_heads * hd, d, bias=False)
        if cfg.qk_norm:
            self.q_norm = RMSNorm(hd, cfg.rms_norm_eps)
            self.k_norm = RMSNorm(hd, cfg.rms_norm_eps)
        else:
            self.q_norm = None
            self.k_norm = None


class Qwen3MLP(nn.Module):
    def __init__(self, cfg: Qwen3Config) -> None:
        super().__init__()
        d, f = cfg.hidden_size, cfg.intermediate_size
        self.gate_proj = nn.Linear(d, f, bias=False)
        self.up_proj = nn.Linear(d, f, bias=False)
        self.down_proj = nn.Linear(f, d, bias=False)


class Qwen3DecoderLayer(nn.Module):
    layer_kind = "full_attention"

    def __init__(self, cfg: Qwen3Config, layer_idx: int) -> None:
        super().__init__()
        self.self_attn = Qwen3Attention(cfg, layer_idx)
        self.mlp = Qwen3MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class Qwen3Model(nn.Module):
    def __init__(self, cfg: Qwen3Config) -> None:
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(Qwen3DecoderLayer(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class Qwen3ForCausalLM(nn.Module):
    """A Qwen3 causal LM whose layers run on this package's native ops."""

    def __init__(self, cfg: Qwen3Config, *, init: bool = True) -> None:
        super().__init__()
        self.config = cfg
        self.model = Qwen3Model(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        if init:
            self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self) -> None:
        """N(0, initializer_range) for matrices, ones for norm weights."""
        std = self.config.initializer_range
        for name, p in self.named_parameters():
            if name.endswith("norm.weight") or "layernorm" in name:
                p.fill_(1.0)
            else:
                p.normal_(0.0, std)

    def forward(
        self,
        input_ids: torch.Tensor,
        position_ids: torch.Tensor | None = None,
    ) -> torch.Tensor:
        """Full-causal logits for a single sequence ``input_ids`` of shape [T] or [1, T]."""
        from thundersync_b200.engine.layers import full_causal_logits

        return full_causal_logits(self, input_ids, position_ids)


def build_qwen3(name_or_cfg: str | Qwen3Config, *, device=None, dtype=None, seed: int | None = None):
    """Random-init model of a named preset (see ``PRESETS``) or config."""
    cfg = PRESETS[name_or_cfg] if isinstance(name_or_cfg, str) else name_or_cfg
    if seed is not None:
        torch.manual_seed(seed)
    with torch.device(device or "cpu"):
        model = Qwen3ForCausalLM(cfg)
    if dtype is not None:
        model.to(dtype=dtype)
    return model


def flops_per_token(cfg: Qwen3Config) -> float:
    """Dense forward FLOPs per token of the matrices (2 * params touched)."""
    d, f = cfg.hidden_size, cfg.intermediate_size
    hq, hk, hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    per_layer = d * hq * hd + 2 * d * hk * hd + hq * hd * d + 3 * d * f
    return 2.0 * (cfg.num_hidden_layers * per_layer + cfg.vocab_size * d)
