"""LoRA adapters: op numerics, deterministic init, PEFT-format files, streamed GRPO gradients.

Reference behaviour: src/thundersync/policy_model.py:240-290 (apply_lora:
seeded, fp32 adapters, caller RNG untouched) and tests/test_policy_model.py;
fused LoRA backward formulas of src/thundersync/accel/fused_lora.py:30-50.
"""

from __future__ import annotations

import json

import pytest
import torch
import torch.nn.functional as F

from tests.grpo_fixtures import EPS, advantages, build_model, make_batch
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward
from thundersync_b200.models.io import load_snapshot, save_snapshot
from thundersync_b200.models.lora import LoRALinear, adapter_state_dict, load_adapter, merged_state_dict
from thundersync_b200.ops.lora import lora_linear
from thundersync_b200.policy_model import (LORA_INIT_SEED, STANDARD_LORA_TARGETS, apply_lora,
                                           lora_target_modules)


def test_lora_linear_value_and_gradient():
    torch.manual_seed(0)
    base = torch.nn.Linear(24, 40, bias=False)
    mod = LoRALinear(base, 4, 8.0)
    with torch.no_grad():
        mod.lora_B["default"].weight.normal_()
    x = torch.randn(7, 24, requires_grad=True)
    y = lora_linear(x, mod)
    a, b = mod.lora_A["default"].weight, mod.lora_B["default"].weight
    ref = F.linear(x, base.weight) + 2.0 * F.linear(F.linear(x, a), b)
    assert torch.allclose(y, ref, atol=1e-5)
    dy = torch.randn_like(y)
    gx, ga, gb = torch.autograd.grad(y, (x, a, b), dy)
    rx, ra, rb = torch.autograd.grad(ref, (x, a, b), dy)
    for got, want in ((gx, rx), (ga, ra), (gb, rb)):
        assert torch.allclose(got, want, atol=1e-5)
    assert base.weight.grad is None


def test_apply_lora_deterministic_and_rng_untouched():
    torch.manual_seed(123)
    before = torch.random.get_rng_state()
    m1 = build_model(0)
    m2 = build_model(0)
    torch.random.set_rng_state(before)
    _, inner1 = apply_lora(m1, rank=4, alpha=8)
    after = torch.random.get_rng_state()
    assert torch.equal(before, after)
    _, inner2 = apply_lora(m2, rank=4, alpha=8)
    s1, s2 = adapter_state_dict(inner1), adapter_state_dict(inner2)
    assert s1.keys() == s2.keys() and len(s1) == 2 * 7 * len(inner1.model.layers)
    for k in s1:
        assert torch.equal(s1[k], s2[k])
        assert s1[k].dtype == torch.float32
    trainable = [n for n, p in inner1.named_parameters() if p.requires_grad]
    assert trainable and all(".lora_" in n for n in trainable)
    assert lora_target_modules(build_model(0)) == STANDARD_LORA_TARGETS
    # the first adapter's A matrix is the seeded generator's draw after the two constructor draws
    torch.manual_seed(LORA_INIT_SEED)
    first = inner1.model.layers[0].self_attn.q_proj
    probe = LoRALinear(torch.nn.Linear(first.in_features, first.out_features, bias=False), 4, 8.0)
    assert probe.lora_A["default"].weight.shape == first.lora_A["default"].weight.shape


def test_adapter_file_roundtrip(tmp_path):
    wrapper, inner = apply_lora(build_model(0), rank=4, alpha=8)
    with torch.no_grad():
        for n, p in inner.named_parameters():
            if "lora_B" in n:
                p.normal_()
    wrapper.save_pretrained(tmp_path)
    cfg = json.loads((tmp_path / "adapter_config.json").read_text())
    assert cfg["r"] == 4 and cfg["lora_alpha"] == 8 and cfg["peft_type"] == "LORA"
    _, other = apply_lora(build_model(0), rank=4, alpha=8)
    load_adapter(other, tmp_path)
    a, b = adapter_state_dict(inner), adapter_state_dict(other)
    assert all(torch.equal(a[k], b[k]) for k in a)
    key = next(iter(a))
    assert key.startswith("base_model.model.model.layers.0.")


def test_merged_state_dict_matches_adapted_forward(tmp_path):
    model = build_model(0)
    _, inner = apply_lora(model, rank=4, alpha=8)
    with torch.no_grad():
        for n, p in inner.named_parameters():
            if "lora_B" in n:
                p.normal_(0, 0.05)
    merged = merged_state_dict(inner)
    assert not any("lora" in k or "base_layer" in k for k in merged)
    plain = build_model(1)
    plain.load_state_dict(merged)
    prompt = list(range(12))
    turns = [([5, 6, 7, 8], [True] * 4)]
    with torch.no_grad():
        lp_a = reference_logprobs(inner, prompt, turns)
        lp_b = reference_logprobs(plain, prompt, turns)
    assert torch.allclose(lp_a, lp_b, atol=1e-4)
    save_snapshot(plain, tmp_path / "snap")
    back = load_snapshot(tmp_path / "snap", dtype=torch.float32)
    for k, v in plain.state_dict().items():
        assert torch.equal(back.state_dict()[k], v), k


def test_streamed_grpo_lora_gradient_matches_reference():
    batch, order = make_batch(seed=3, groups=2, per_group=3, lo=4, hi=10)
    model = build_model(0)
    _, inner = apply_lora(model, rank=4, alpha=8)
    with torch.no_grad():
        for n, p in inner.named_parameters():
            if "lora_B" in n:
                p.normal_(0, 0.05)
    # oracle: full-batch reward-weighted logprob gradient
    inner.zero_grad(set_to_none=True)
    total = 0.0
    for g, prompt, trajs in batch:
        adv = advantages([r for _, _, r in trajs])
        for (tid, turns, _), a in zip(trajs, adv):
            total = total + a * reference_logprobs(inner, prompt, turns).sum()
    total.backward()
    ref = {n: p.grad.clone() for n, p in inner.named_parameters() if p.requires_grad}
    inner.zero_grad(set_to_none=True)
    run = StreamingRun(inner, boundary_cut=True, stream_turns=False)
    bw = RewardLinearBackward(run, inner, eps=EPS)
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for g, (tid, turns, reward) in order:
        for tk, sc in turns:
            run.append_turn(g, tid, tk, sc)
        bw.close_trajectory(tid, reward)
    for g, _, _ in batch:
        bw.close_group(g)
    bw.assert_safe_to_step()
    for n, p in inner.named_parameters():
        if not p.requires_grad:
            assert p.grad is None, n
            continue
        assert p.grad is not None, n
        assert torch.allclose(p.grad, ref[n], atol=2e-5, rtol=1e-4), (n, (p.grad - ref[n]).abs().max())
