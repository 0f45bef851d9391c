"""Hybrid GDN / gated-attention model: executor vs an independent torch reference (CPU fp32)."""

from __future__ import annotations

import copy
import math
import random

import torch
import torch.nn.functional as F

from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward
from thundersync_b200.models.hybrid import HYBRID_PRESETS, HybridForCausalLM
from thundersync_b200.ops.gdn import causal_conv1d_reference, causal_conv1d_silu, gated_delta_rule, gated_delta_rule_reference


def _model(seed=0):
    torch.manual_seed(seed)
    return HybridForCausalLM(HYBRID_PRESETS["hybrid-tiny"])


def _rms_unit(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * (1 + w.float())).to(x.dtype)


def _rms(x, w, eps):
    xf = x.float()
    n = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)
    return (w.float() * n.float()).to(x.dtype)


def reference_hidden(model, ids):
    """Monolithic forward in plain torch, HF Qwen3.5-text semantics."""
    cfg = model.config
    t = ids.shape[0]
    eps = cfg.rms_norm_eps
    h = model.model.embed_tokens.weight[ids]
    pos = torch.arange(t)
    rd = cfg.rotary_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, rd, 2).float() / rd))
    fr = pos.float()[:, None] * inv[None]
    emb = torch.cat((fr, fr), -1)
    cos, sin = emb.cos()[:, None], emb.sin()[:, None]

    def rope(x):
        xr, xp = x[..., :rd], x[..., rd:]
        hh = rd // 2
        rot = torch.cat((-xr[..., hh:], xr[..., :hh]), -1)
        return torch.cat((xr * cos + rot * sin, xp), -1)

    for layer in model.model.layers:
        x = _rms_unit(h, layer.input_layernorm.weight, eps)
        if layer.layer_kind == "linear_attention":
            m = layer.linear_attn
            mixed = F.linear(x, m.in_proj_qkv.weight)
            z = F.linear(x, m.in_proj_z.weight)
            b = F.linear(x, m.in_proj_b.weight)
            a = F.linear(x, m.in_proj_a.weight)
            conv = F.conv1d(mixed.t()[None], m.conv1d.weight, padding=m.conv_kernel_size - 1, groups=m.conv_dim)
            qkv = F.silu(conv[0, :, :t]).t()
            q = qkv[:, : m.key_dim].reshape(t, m.num_k_heads, m.head_k_dim)
            k = qkv[:, m.key_dim : 2 * m.key_dim].reshape(t, m.num_k_heads, m.head_k_dim)
            v = qkv[:, 2 * m.key_dim :].reshape(t, m.num_v_heads, m.head_v_dim)
            rep = m.num_v_heads // m.num_k_heads
            q, k = q.repeat_interleave(rep, 1), k.repeat_interleave(rep, 1)
            beta = b.sigmoid()
            g = -m.A_log.float().exp() * F.softplus(a.float() + m.dt_bias)
            core, _ = gated_delta_rule_reference(q, k, v, g, beta)
            core = _rms(core.reshape(-1, m.head_v_dim), m.norm.weight, eps) * F.silu(z.reshape(-1, m.head_v_dim))
            h = h + F.linear(core.reshape(t, -1), m.out_proj.weight)
        else:
            sa = layer.self_attn
            hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
            qg = F.linear(x, sa.q_proj.weight).view(t, hq, 2 * d)
            q, gate = qg[..., :d], qg[..., d:].reshape(t, hq * d)
            q = rope(_rms_unit(q, sa.q_norm.weight, eps))
            k = rope(_rms_unit(F.linear(x, sa.k_proj.weight).view(t, hkv, d), sa.k_norm.weight, eps))
            v = F.linear(x, sa.v_proj.weight).view(t, hkv, d)
            gq = hq // hkv
            kf, vf = k.repeat_interleave(gq, 1).transpose(0, 1), v.repeat_interleave(gq, 1).transpose(0, 1)
            sc = q.transpose(0, 1) @ kf.transpose(1, 2) / math.sqrt(d)
            sc = sc.masked_fill(~torch.ones(t, t, dtype=torch.bool).tril(), float("-inf"))
            o = (sc.softmax(-1) @ vf).transpose(0, 1).reshape(t, hq * d) * torch.sigmoid(gate)
            h = h + F.linear(o, sa.o_proj.weight)
        x = _rms_unit(h, layer.post_attention_layernorm.weight, eps)
        mlp = layer.mlp
        h = h + F.linear(F.silu(F.linear(x, mlp.gate_proj.weight)) * F.linear(x, mlp.up_proj.weight), mlp.down_proj.weight)
    return _rms_unit(h, model.model.norm.weight, eps)


def _lp(model, prompt, turns):
    toks = prompt + [t for tk, _ in turns for t in tk]
    sc = [False] * len(prompt) + [s for _, ss in turns for s in ss]
    h = reference_hidden(model, torch.tensor(toks))
    lp = torch.log_softmax(h @ model.lm_head.weight.t(), -1)
    idx = [i for i, s in enumerate(sc) if s]
    return lp[torch.tensor([i - 1 for i in idx])].gather(-1, torch.tensor([toks[i] for i in idx])[:, None]).squeeze(-1)


def test_conv1d_tail_chaining_matches_monolithic():
    torch.manual_seed(0)
    x = torch.randn(20, 6)
    w = torch.randn(6, 4)
    full, _ = causal_conv1d_reference(x, w, None)
    y1, t1 = causal_conv1d_silu(x[:7], w, None)
    y2, _ = causal_conv1d_silu(x[7:], w, t1)
    torch.testing.assert_close(torch.cat((y1, y2)), full)


def test_delta_rule_state_chaining():
    torch.manual_seed(1)
    t, h, dk, dv = 12, 2, 8, 8
    q, k, v = torch.randn(t, h, dk), torch.randn(t, h, dk), torch.randn(t, h, dv)
    g, beta = -torch.rand(t, h), torch.rand(t, h)
    o, s = gated_delta_rule(q, k, v, g, beta)
    o1, s1 = gated_delta_rule(q[:5], k[:5], v[:5], g[:5], beta[:5])
    o2, s2 = gated_delta_rule(q[5:], k[5:], v[5:], g[5:], beta[5:], s1)
    torch.testing.assert_close(torch.cat((o1, o2)), o)
    torch.testing.assert_close(s2, s)


def test_hybrid_streamed_logprobs_and_grpo_gradient_match_reference():
    model = _model(2)
    rng = random.Random(3)
    prompt = [rng.randrange(512) for _ in range(9)]
    trajs = []
    for tid in range(3):
        turns = []
        for _ in range(2):
            a = [rng.randrange(512) for _ in range(rng.randint(2, 5))]
            o = [rng.randrange(512) for _ in range(2)]
            turns.append((a + o, [True] * len(a) + [False] * len(o)))
        trajs.append((tid, turns, float(tid % 2)))
    ref_model = copy.deepcopy(model)
    r = torch.tensor([x for _, _, x in trajs], dtype=torch.float64)
    mean, std = float(r.mean()), float(r.std(unbiased=False)) + 1e-6
    total = sum(((rw - mean) / std) * _lp(ref_model, prompt, turns).sum() for _, turns, rw in trajs)
    total.backward()
    run = StreamingRun(model, boundary_cut=True)
    bw = RewardLinearBackward(run, model)
    bw.open_group(0, prompt, [t for t, _, _ in trajs])
    for tid, turns, rw in trajs:
        for tk, sc in turns:
            run.append_turn(0, tid, tk, sc)
        torch.testing.assert_close(run.logprobs(tid), _lp(ref_model, prompt, turns).detach(), rtol=1e-4, atol=1e-5)
        bw.close_trajectory(tid, rw)
    bw.close_group(0)
    bw.assert_safe_to_step()
    for (n, p), (_, q) in zip(model.named_parameters(), ref_model.named_parameters()):
        torch.testing.assert_close(p.grad, q.grad, rtol=5e-4, atol=5e-6, msg=n)
