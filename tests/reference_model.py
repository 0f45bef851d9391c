"""Independent plain-torch Qwen3 forward used as the oracle in tests.

It reads the same parameters by their HF names but uses none of
``thundersync_b200.ops``: dense causal attention with a full mask, explicit
RMSNorm and rotate-half RoPE, full-vocabulary log-softmax. Mirrors the role of
the reference's tests/reference_logprobs.py.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _rms(x, w, eps):
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return (w.float() * n.float()).to(x.dtype)


def _lin(x, mod):
    """``mod(x)`` for a plain or LoRA (PEFT-layout) linear, in plain torch."""
    base = getattr(mod, "base_layer", None)
    if base is None:
        return F.linear(x, mod.weight)
    a, b = mod.lora_A["default"].weight, mod.lora_B["default"].weight
    low = F.linear(F.linear(x.to(a.dtype), a), b) * mod.scaling["default"]
    return (F.linear(x, base.weight).to(low.dtype) + low).to(x.dtype)


def _rope(x, pos, theta):
    d = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, d, 2, dtype=torch.int64).float() / d))
    fr = pos.float()[:, None] * inv[None].to(x.device)
    emb = torch.cat((fr, fr), -1)
    cos, sin = emb.cos()[:, None], emb.sin()[:, None]
    h = d // 2
    rot = torch.cat((-x[..., h:], x[..., :h]), -1)
    return (x.float() * cos + rot.float() * sin).to(x.dtype)


def hidden_states(model, ids: torch.Tensor) -> torch.Tensor:
    cfg = model.config
    hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    eps, theta = cfg.rms_norm_eps, cfg.rope_theta
    t = ids.shape[0]
    pos = torch.arange(t, device=ids.device)
    h = model.model.embed_tokens.weight[ids]
    mask = torch.ones(t, t, dtype=torch.bool, device=ids.device).tril()
    for layer in model.model.layers:
        sa = layer.self_attn
        x = _rms(h, layer.input_layernorm.weight, eps)
        q = _lin(x, sa.q_proj).view(t, hq, d)
        k = _lin(x, sa.k_proj).view(t, hkv, d)
        v = _lin(x, sa.v_proj).view(t, hkv, d)
        if sa.q_norm is not None:
            q = _rms(q, sa.q_norm.weight, eps)
            k = _rms(k, sa.k_norm.weight, eps)
        q, k = _rope(q, pos, theta), _rope(k, pos, theta)
        g = hq // hkv
        kf = k.repeat_interleave(g, 1).transpose(0, 1).float()
        vf = v.repeat_interleave(g, 1).transpose(0, 1).float()
        s = q.transpose(0, 1).float() @ kf.transpose(1, 2) / math.sqrt(d)
        s = s.masked_fill(~mask, float("-inf"))
        o = (torch.softmax(s, -1) @ vf).transpose(0, 1).reshape(t, hq * d).to(h.dtype)
        h = h + _lin(o, sa.o_proj)
        x = _rms(h, layer.post_attention_layernorm.weight, eps)
        gt, up = _lin(x, layer.mlp.gate_proj), _lin(x, layer.mlp.up_proj)
        a = (F.silu(gt.float()) * up.float()).to(h.dtype)
        h = h + _lin(a, layer.mlp.down_proj)
    return _rms(h, model.model.norm.weight, eps)


def reference_logprobs(model, prompt: list[int], turns: list[tuple[list[int], list[bool]]]) -> torch.Tensor:
    """Scored-token log-probs of one trajectory, computed alone with full logits."""
    dev = model.lm_head.weight.device
    toks = list(prompt)
    scored = [False] * len(prompt)
    for tk, sc in turns:
        toks += list(tk)
        scored += list(sc)
    ids = torch.tensor(toks, device=dev)
    h = hidden_states(model, ids)
    logits = h.float() @ model.lm_head.weight.float().t()
    lp = torch.log_softmax(logits, -1)
    idx = [i for i, s in enumerate(scored) if s and i > 0]
    if not idx:
        return lp.new_zeros(0)
    src = torch.tensor([i - 1 for i in idx], device=dev)
    tgt = torch.tensor([toks[i] for i in idx], device=dev)
    return lp[src].gather(-1, tgt[:, None]).squeeze(-1)
