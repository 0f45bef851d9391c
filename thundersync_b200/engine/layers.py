"""Layer executor: runs a Qwen3-family model on this package's native ops.

The executor reads parameters by their Hugging Face names (so it drives this
package's own ``Qwen3ForCausalLM``/``HybridForCausalLM`` and, structurally,
an HF Qwen3 module too) and runs one *pack* of segments per call. A segment
is a contiguous run of new tokens plus the ancestor state it attends to:
per attention layer a list of K/V chunks, per linear-attention layer the
parent's (conv tail, recurrent state). All segments of a pack share the dense
GEMMs (one QKV GEMM, one gate/up GEMM per layer over the concatenated tokens);
attention and the recurrent scan run per segment over each one's own chain.

This replaces the reference's HF ``AttentionInterface`` hook plus its
per-layer checkpoint wrappers (src/thundersync/engine/streaming.py:1439-1539,
:2043-2100) with one explicit executor whose per-layer K/V outputs are
ordinary autograd tensors.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

import torch

from thundersync_b200.ops.attention import chunked_attention
from thundersync_b200.ops.packed_attention import packed_attention
from thundersync_b200.ops.embedding import embedding
from thundersync_b200.ops.linear import linear
from thundersync_b200.ops.norm import rms_norm
from thundersync_b200.ops.rope import qk_norm_rope, rope_inv_freq
from thundersync_b200.ops.swiglu import swiglu

__all__ = ["ModelSpec", "spec_of", "Executor", "Segment", "full_causal_logits", "executor_for"]


@dataclass(frozen=True)
class ModelSpec:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv: int
    head_dim: int
    eps: float
    rope_theta: float
    vocab: int
    tied: bool
    qk_norm: bool
    kinds: tuple[str, ...]
    attn_gate: bool = False  # hybrid full-attention layers gate their output
    rotary_dim: int = 0  # dims of each head that rotate (0 = all)
    unit_norm: bool = False  # zero-centred (1 + w) RMSNorms (Qwen3.5)

    @property
    def attention_layers(self) -> list[int]:
        return [i for i, k in enumerate(self.kinds) if k == "full_attention"]

    @property
    def linear_layers(self) -> list[int]:
        return [i for i, k in enumerate(self.kinds) if k == "linear_attention"]


def _cfg_get(cfg: Any, name: str, default: Any = None) -> Any:
    value = getattr(cfg, name, None)
    return default if value is None else value


def spec_of(model: torch.nn.Module) -> ModelSpec:
    cfg = model.config
    hidden = cfg.hidden_size
    heads = cfg.num_attention_heads
    head_dim = _cfg_get(cfg, "head_dim", hidden // heads)
    theta = getattr(cfg, "rope_theta", None)
    if theta is None:
        rope = _cfg_get(cfg, "rope_parameters", {}) or {}
        theta = rope.get("rope_theta", 10000.0) if isinstance(rope, dict) else 10000.0
    layers = model.model.layers
    kinds = []
    for i, layer in enumerate(layers):
        kind = getattr(layer, "layer_kind", None) or getattr(layer, "layer_type", None)
        if kind is None:
            types = _cfg_get(cfg, "layer_types", None)
            kind = types[i] if types else "full_attention"
        kinds.append(kind)
    first_attn = next((layers[i] for i, k in enumerate(kinds) if k == "full_attention"), None)
    qk_norm = bool(first_attn is not None and getattr(first_attn.self_attn, "q_norm", None) is not None)
    attn_gate = False
    if first_attn is not None:
        qw = _weight(first_attn.self_attn.q_proj)
        attn_gate = qw.shape[0] == 2 * heads * head_dim
    factor = float(_cfg_get(cfg, "partial_rotary_factor", 1.0))
    return ModelSpec(
        n_layers=len(layers),
        hidden=hidden,
        n_heads=heads,
        n_kv=cfg.num_key_value_heads,
        head_dim=head_dim,
        eps=float(_cfg_get(cfg, "rms_norm_eps", 1e-6)),
        rope_theta=float(theta),
        vocab=cfg.vocab_size,
        tied=bool(_cfg_get(cfg, "tie_word_embeddings", False)),
        qk_norm=qk_norm,
        kinds=tuple(kinds),
        attn_gate=attn_gate,
        rotary_dim=int(head_dim * factor),
        unit_norm=_is_unit(model.model.norm),
    )


def _is_unit(norm_module) -> bool:
    return bool(getattr(norm_module, "unit_offset", False)) or type(norm_module).__name__ in (
        "Qwen3_5RMSNorm", "Qwen3NextRMSNorm")


@dataclass
class Segment:
    """New tokens ``[start, start+length)`` of a pack and the state they attend to.

    ``past[layer]`` is, for attention layers, ``(k_chunks, v_chunks)``: lists
    of [S_i, Hkv, d] tensors, ancestors first. For linear-attention layers it
    is ``(conv_tail, state)`` (either may be None for a root).
    """

    start: int
    length: int
    past: list[Any] = field(default_factory=list)
    key_ranges: list[tuple[int, int]] = field(default_factory=list)
    """Ancestor spans inside the same pack (forest execution): each layer reads
    ``k[s:e]``/``v[s:e]`` of the pack's own projections after ``past``."""


def _weight(mod: torch.nn.Module) -> torch.Tensor:
    base = getattr(mod, "base_layer", None)
    return (base if base is not None else mod).weight


def _is_lora(mod: torch.nn.Module) -> bool:
    return getattr(mod, "lora_A", None) is not None and getattr(mod, "base_layer", None) is not None


class Executor:
    """Runs embeddings, layers and the final norm of one model."""

    def __init__(self, model: torch.nn.Module, arena=None) -> None:
        self.model = model
        self.spec = spec_of(model)
        self.arena = arena
        self._inv_freq: dict[torch.device, torch.Tensor] = {}
        # one autograd node per dense layer (engine/dense_layer.py); False runs op by op
        self.fused_layers = True
        self._dense_ok: dict[int, bool] = {}

    # ------------------------------------------------------------ pieces
    def inv_freq(self, device: torch.device) -> torch.Tensor:
        t = self._inv_freq.get(device)
        if t is None:
            t = rope_inv_freq(self.spec.rotary_dim or self.spec.head_dim, self.spec.rope_theta, device)
            self._inv_freq[device] = t
        return t

    def embed(self, ids: torch.Tensor) -> torch.Tensor:
        return embedding(ids, self.model.model.embed_tokens.weight)

    def norm(self, mod, x: torch.Tensor) -> torch.Tensor:
        eps = getattr(mod, "variance_epsilon", None) or getattr(mod, "eps", None) or self.spec.eps
        return rms_norm(x, mod.weight, eps, unit_offset=_is_unit(mod))

    def final_norm(self, h: torch.Tensor) -> torch.Tensor:
        return self.norm(self.model.model.norm, h)

    def head_weight(self) -> torch.Tensor:
        return _weight(self.model.lm_head)

    def proj(self, x: torch.Tensor, mods: list[torch.nn.Module]) -> torch.Tensor:
        if any(_is_lora(m) for m in mods):
            from thundersync_b200.ops.lora import lora_linear

            outs = [lora_linear(x, m) if _is_lora(m) else linear(x, [_weight(m)]) for m in mods]
            return outs[0] if len(outs) == 1 else torch.cat(outs, -1)
        return linear(x, [_weight(m) for m in mods], self.arena)

    # ------------------------------------------------------------ layers
    def _plain_dense(self, layer) -> bool:
        """A Qwen3 layer the single-node layer op covers (no gate, no LoRA, weight-scaled norms)."""
        key = id(layer)
        got = self._dense_ok.get(key)
        if got is None:
            sa, mlp = layer.self_attn, layer.mlp
            mods = [sa.q_proj, sa.k_proj, sa.v_proj, sa.o_proj, mlp.gate_proj, mlp.up_proj, mlp.down_proj]
            norms = [layer.input_layernorm, layer.post_attention_layernorm]
            qn = getattr(sa, "q_norm", None)
            if qn is not None:
                norms.append(qn)
            got = (not self.spec.attn_gate and not any(_is_lora(m) for m in mods)
                   and not any(_is_unit(n) for n in norms))
            self._dense_ok[key] = got
        return got

    def attention_layer(self, i: int, h: torch.Tensor, pos: torch.Tensor, segs: list[Segment]):
        spec = self.spec
        layer = self.model.model.layers[i]
        if self.fused_layers and self._plain_dense(layer):
            from thundersync_b200.engine.dense_layer import dense_layer

            return dense_layer(self, i, h, pos, segs)
        sa = layer.self_attn
        hq, hkv, d = spec.n_heads, spec.n_kv, spec.head_dim
        x = self.norm(layer.input_layernorm, h)
        if spec.attn_gate:
            # Hybrid gated attention: q_proj emits [q, gate] per head.
            qg = self.proj(x, [sa.q_proj])
            t = qg.shape[0]
            qg = qg.view(t, hq, 2 * d)
            q_raw, gate = qg[..., :d].reshape(t, hq * d), qg[..., d:].reshape(t, hq * d)
            kv = self.proj(x, [sa.k_proj, sa.v_proj])
            qkv = torch.cat((q_raw, kv), -1)
        else:
            qkv = self.proj(x, [sa.q_proj, sa.k_proj, sa.v_proj])
            gate = None
        qn = getattr(sa, "q_norm", None)
        kn = getattr(sa, "k_norm", None)
        q, k, v = qk_norm_rope(
            qkv, None if qn is None else qn.weight, None if kn is None else kn.weight,
            pos, self.inv_freq(h.device), hq, hkv, d, spec.eps, unit_offset=qn is not None and _is_unit(qn),
        )
        scale = 1.0 / math.sqrt(d)
        new_state = [(k[seg.start:seg.start + seg.length], v[seg.start:seg.start + seg.length]) for seg in segs]
        if q.is_cuda and (len(segs) > 1 or segs[0].key_ranges):
            # every segment in one packed launch (shared ancestor chunks stored and differentiated once)
            meta, pk, pv = [], [], []
            for seg in segs:
                ks, vs = seg.past[i] if seg.past and seg.past[i] is not None else ([], [])
                pk.extend(ks)
                pv.extend(vs)
                meta.append((seg.start, seg.start + seg.length, len(ks), tuple(seg.key_ranges)))
            o = packed_attention(q, k, v, meta, pk, pv, scale)
        else:
            outs = []
            for seg in segs:
                s0, s1 = seg.start, seg.start + seg.length
                ks, vs = seg.past[i] if seg.past and seg.past[i] is not None else ([], [])
                if seg.key_ranges:
                    ks = [*ks, *(k[a:b] for a, b in seg.key_ranges)]
                    vs = [*vs, *(v[a:b] for a, b in seg.key_ranges)]
                outs.append(chunked_attention(q[s0:s1], [*ks, k[s0:s1]], [*vs, v[s0:s1]], scale))
            covered = sum(seg.length for seg in segs)
            if covered < qkv.shape[0]:  # pack padding rows: no attention output
                outs.append(q.new_zeros(qkv.shape[0] - covered, hq, d))
            o = outs[0] if len(outs) == 1 else torch.cat(outs, 0)
        o = o.reshape(o.shape[0], hq * d)
        if gate is not None:
            o = o * torch.sigmoid(gate.float()).to(o.dtype)
        h = h + self.proj(o, [sa.o_proj])
        h = self.mlp(layer, h)
        return h, new_state

    def mlp(self, layer, h: torch.Tensor) -> torch.Tensor:
        mlp = layer.mlp
        x = self.norm(layer.post_attention_layernorm, h)
        gu = self.proj(x, [mlp.gate_proj, mlp.up_proj])
        return h + self.proj(swiglu(gu), [mlp.down_proj])

    def linear_layer(self, i: int, h: torch.Tensor, pos: torch.Tensor, segs: list[Segment]):
        from thundersync_b200.models.hybrid import gated_deltanet_layer

        layer = self.model.model.layers[i]
        return gated_deltanet_layer(self, layer, i, h, segs)

    def run(self, ids: torch.Tensor, pos: torch.Tensor, segs: list[Segment], *, norm: bool = True):
        """Forward a pack. Returns (hidden [T, D], per-segment per-layer new state)."""
        h = self.embed(ids)
        states: list[list[Any]] = [[None] * self.spec.n_layers for _ in segs]
        for i, kind in enumerate(self.spec.kinds):
            if kind == "full_attention":
                h, new = self.attention_layer(i, h, pos, segs)
            else:
                h, new = self.linear_layer(i, h, pos, segs)
            for j, st in enumerate(new):
                states[j][i] = st
        if norm:
            h = self.final_norm(h)
        return h, states


def executor_for(model: torch.nn.Module, arena=None) -> Executor:
    ex = getattr(model, "_ts_executor", None)
    if ex is None or ex.arena is not arena:
        ex = Executor(model, arena)
        try:
            object.__setattr__(model, "_ts_executor", ex)
        except Exception:
            pass
    return ex


def full_causal_logits(model, input_ids: torch.Tensor, position_ids: torch.Tensor | None = None):
    """Plain causal forward of one sequence -> fp32 logits [T, V] (tests, oracle)."""
    ids = input_ids.reshape(-1)
    t = ids.shape[0]
    pos = torch.arange(t, device=ids.device) if position_ids is None else position_ids.reshape(-1)
    ex = Executor(model)
    h, _ = ex.run(ids, pos, [Segment(0, t, [])])
    w = ex.head_weight()
    if h.dtype == torch.bfloat16 and h.is_cuda:
        from thundersync_b200.ops.gemm import gemm

        return gemm(h, w, out_dtype=torch.float32)
    return h.float() @ w.float().t()
