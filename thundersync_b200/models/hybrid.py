"""Hybrid linear / full-attention decoder (Qwen3.5-text layout) on native ops.

Layers repeat ``full_attention_interval - 1`` Gated DeltaNet layers and one
gated full-attention layer. Parameter names follow Hugging Face's Qwen3.5
text model (``model.layers.N.linear_attn.{in_proj_qkv,in_proj_z,in_proj_b,
in_proj_a,conv1d,dt_bias,A_log,norm,out_proj}``, ``self_attn.{q,k,v,o}_proj``
with a doubled ``q_proj`` carrying the output gate, zero-centred
``(1 + w)`` RMSNorms), so snapshots load with identical keys (reference:
src/thundersync/policy_model.py:90-179 loads that class; the streaming layer
it runs is reference src/thundersync/engine/streaming.py:1918-2040).

A linear-attention layer carries two gradient channels across segments, the
recurrent state [H, dk, dv] (fp32) and the conv tail [K-1, conv_dim]; the
executor treats them exactly as attention layers treat ancestor K/V.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass, field, replace
from typing import Any

import torch
import torch.nn.functional as F
from torch import nn

from thundersync_b200.ops.gdn import causal_conv1d_silu, gated_delta_rule
from thundersync_b200.ops.norm import rms_norm

__all__ = ["HybridConfig", "HybridForCausalLM", "HYBRID_PRESETS", "gated_deltanet_layer"]


@dataclass(frozen=True)
class HybridConfig:
    vocab_size: int = 151936
    hidden_size: int = 2048
    intermediate_size: int = 5632
    num_hidden_layers: int = 48
    full_attention_interval: int = 4
    num_attention_heads: int = 16
    num_key_value_heads: int = 2
    head_dim: int = 256
    partial_rotary_factor: float = 0.25
    rope_theta: float = 10_000_000.0
    rms_norm_eps: float = 1e-6
    linear_conv_kernel_dim: int = 4
    linear_key_head_dim: int = 128
    linear_value_head_dim: int = 128
    linear_num_key_heads: int = 16
    linear_num_value_heads: int = 16
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 65536
    initializer_range: float = 0.02
    attn_output_gate: bool = True
    model_type: str = "qwen3_5_text"
    extra: dict = field(default_factory=dict, compare=False, hash=False)

    @property
    def layer_types(self) -> list[str]:
        return ["full_attention" if (i + 1) % self.full_attention_interval == 0 else "linear_attention"
                for i in range(self.num_hidden_layers)]

    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    def to_dict(self) -> dict[str, Any]:
        out = asdict(self)
        out.pop("extra")
        out.update(self.extra)
        out["layer_types"] = self.layer_types
        return out

    def with_(self, **changes: Any) -> "HybridConfig":
        return replace(self, **changes)


HYBRID_PRESETS: dict[str, HybridConfig] = {
    # 48 layers of 3x GDN + 1x gated attention.
    "hybrid-48l": HybridConfig(),
    "hybrid-tiny": HybridConfig(
        vocab_size=512, hidden_size=64, intermediate_size=128, num_hidden_layers=4, num_attention_heads=4,
        num_key_value_heads=2, head_dim=32, partial_rotary_factor=0.5, linear_key_head_dim=16,
        linear_value_head_dim=16, linear_num_key_heads=2, linear_num_value_heads=4, max_position_embeddings=4096,
    ),
}


class ZeroCenteredRMSNorm(nn.Module):
    """RMSNorm whose weight is stored zero-centred and applied as ``1 + w``."""

    unit_offset = True

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.zeros(dim))
        self.eps = eps
        self.variance_epsilon = eps

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return rms_norm(x, self.weight, self.eps, unit_offset=True)


class GatedRMSNorm(nn.Module):
    """Norm before gate: ``w * round(norm(x)) * silu(z)`` (weight stored as-is)."""

    def __init__(self, dim: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.variance_epsilon = eps


class GatedDeltaNet(nn.Module):
    def __init__(self, cfg: HybridConfig, layer_idx: int) -> None:
        super().__init__()
        self.layer_idx = layer_idx
        self.num_v_heads = cfg.linear_num_value_heads
        self.num_k_heads = cfg.linear_num_key_heads
        self.head_k_dim = cfg.linear_key_head_dim
        self.head_v_dim = cfg.linear_value_head_dim
        self.key_dim = self.head_k_dim * self.num_k_heads
        self.value_dim = self.head_v_dim * self.num_v_heads
        self.conv_kernel_size = cfg.linear_conv_kernel_dim
        self.conv_dim = 2 * self.key_dim + self.value_dim
        d = cfg.hidden_size
        # projections first and adjacent, so the arena can run them as one GEMM
        self.in_proj_qkv = nn.Linear(d, self.conv_dim, bias=False)
        self.in_proj_z = nn.Linear(d, self.value_dim, bias=False)
        self.in_proj_b = nn.Linear(d, self.num_v_heads, bias=False)
        self.in_proj_a = nn.Linear(d, self.num_v_heads, bias=False)
        self.conv1d = nn.Conv1d(self.conv_dim, self.conv_dim, bias=False, kernel_size=self.conv_kernel_size,
                                groups=self.conv_dim, padding=self.conv_kernel_size - 1)
        self.dt_bias = nn.Parameter(torch.ones(self.num_v_heads))
        self.A_log = nn.Parameter(torch.empty(self.num_v_heads).uniform_(0, 16).log_())
        self.norm = GatedRMSNorm(self.head_v_dim, cfg.rms_norm_eps)
        self.out_proj = nn.Linear(self.value_dim, d, bias=False)


class GatedAttention(nn.Module):
    def __init__(self, cfg: HybridConfig, layer_idx: int) -> None:
        super().__init__()
        d, hd = cfg.hidden_size, cfg.head_dim
        self.layer_idx = layer_idx
        self.head_dim = hd
        self.q_proj = nn.Linear(d, cfg.num_attention_heads * hd * 2, bias=False)
        self.k_proj = nn.Linear(d, cfg.num_key_value_heads * hd, bias=False)
        self.v_proj = nn.Linear(d, cfg.num_key_value_heads * hd, bias=False)
        self.o_proj = nn.Linear(cfg.num_attention_heads * hd, d, bias=False)
        self.q_norm = ZeroCenteredRMSNorm(hd, cfg.rms_norm_eps)
        self.k_norm = ZeroCenteredRMSNorm(hd, cfg.rms_norm_eps)


class HybridMLP(nn.Module):
    def __init__(self, cfg: HybridConfig) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)


class HybridDecoderLayer(nn.Module):
    def __init__(self, cfg: HybridConfig, layer_idx: int) -> None:
        super().__init__()
        self.layer_kind = cfg.layer_types[layer_idx]
        if self.layer_kind == "linear_attention":
            self.linear_attn = GatedDeltaNet(cfg, layer_idx)
        else:
            self.self_attn = GatedAttention(cfg, layer_idx)
        self.mlp = HybridMLP(cfg)
        self.input_layernorm = ZeroCenteredRMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = ZeroCenteredRMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class HybridModel(nn.Module):
    def __init__(self, cfg: HybridConfig) -> None:
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(HybridDecoderLayer(cfg, i) for i in range(cfg.num_hidden_layers))
        self.norm = ZeroCenteredRMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class HybridForCausalLM(nn.Module):
    """Hybrid GDN / gated-attention causal LM whose layers run on native ops."""

    def __init__(self, cfg: HybridConfig, *, init: bool = True) -> None:
        super().__init__()
        self.config = cfg
        self.model = HybridModel(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)
        if cfg.tie_word_embeddings:
            self.lm_head.weight = self.model.embed_tokens.weight
        if init:
            self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self) -> None:
        std = self.config.initializer_range
        for mod in self.modules():
            if isinstance(mod, ZeroCenteredRMSNorm):
                mod.weight.zero_()
            elif isinstance(mod, GatedRMSNorm):
                mod.weight.fill_(1.0)
            elif isinstance(mod, GatedDeltaNet):
                mod.dt_bias.fill_(1.0)
                mod.A_log.copy_(torch.empty_like(mod.A_log).uniform_(0, 16).log_())
            elif isinstance(mod, (nn.Linear, nn.Embedding, nn.Conv1d)):
                mod.weight.normal_(0.0, std)

    def forward(self, input_ids: torch.Tensor, position_ids: torch.Tensor | None = None) -> torch.Tensor:
        from thundersync_b200.engine.layers import full_causal_logits

        return full_causal_logits(self, input_ids, position_ids)


def gated_deltanet_layer(ex, layer, i: int, h: torch.Tensor, segs):
    """One linear-attention decoder layer over a pack; returns (h, [(state, tail)] per segment)."""
    mix = layer.linear_attn
    eps = ex.spec.eps
    x = rms_norm(h, layer.input_layernorm.weight, eps, unit_offset=True)
    proj = ex.proj(x, [mix.in_proj_qkv, mix.in_proj_z, mix.in_proj_b, mix.in_proj_a])
    cd, vd, hv = mix.conv_dim, mix.value_dim, mix.num_v_heads
    mixed = proj[:, :cd]
    z = proj[:, cd : cd + vd]
    b = proj[:, cd + vd : cd + vd + hv]
    a = proj[:, cd + vd + hv :]
    beta = torch.sigmoid(b.float())
    g = -mix.A_log.float().exp() * F.softplus(a.float() + mix.dt_bias.float())
    weight = mix.conv1d.weight.squeeze(1)
    rep = mix.num_v_heads // mix.num_k_heads
    outs, finals = [], []
    for seg in segs:
        s0, s1 = seg.start, seg.start + seg.length
        past = seg.past[i] if seg.past and seg.past[i] is not None else (None, None)
        state0, tail0 = past
        qkv, tail = causal_conv1d_silu(mixed[s0:s1], weight, tail0)
        t = s1 - s0
        q = qkv[:, : mix.key_dim].reshape(t, mix.num_k_heads, mix.head_k_dim)
        k = qkv[:, mix.key_dim : 2 * mix.key_dim].reshape(t, mix.num_k_heads, mix.head_k_dim)
        v = qkv[:, 2 * mix.key_dim :].reshape(t, mix.num_v_heads, mix.head_v_dim)
        if rep > 1:
            q = q.repeat_interleave(rep, dim=1)
            k = k.repeat_interleave(rep, dim=1)
        core, state = gated_delta_rule(q, k, v, g[s0:s1], beta[s0:s1], state0)
        outs.append(core)
        finals.append((state, tail))
    covered = sum(seg.length for seg in segs)
    if covered < h.shape[0]:  # pack padding rows: no mixer output
        outs.append(outs[0].new_zeros(h.shape[0] - covered, *outs[0].shape[1:]))
    core = outs[0] if len(outs) == 1 else torch.cat(outs, 0)  # [T, Hv, dv]
    t_all = core.shape[0]
    normed = rms_norm(core.reshape(-1, mix.head_v_dim), mix.norm.weight, mix.norm.variance_epsilon)
    gate = F.silu(z.reshape(-1, mix.head_v_dim).float())
    core = (normed.float() * gate).to(h.dtype).reshape(t_all, vd)
    h = h + ex.proj(core, [mix.out_proj])
    h = ex.mlp(layer, h)
    return h, finals
