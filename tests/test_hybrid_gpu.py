"""Hybrid (GDN + gated attention) streamed GRPO on the GPU kernels vs an fp32 plain-torch oracle.

Reference behaviour: Qwen3.5-text hybrid layers on the streaming path
(src/thundersync/engine/streaming.py:1918-2040) and the GRPO gradient
identity of src/thundersync/grpo/reward_linear.py.
"""

from __future__ import annotations

import copy
import random

import pytest
import torch

from tests.test_hybrid import _lp
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward
from thundersync_b200.models.hybrid import HybridConfig, HybridForCausalLM

pytestmark = pytest.mark.gpu

CFG = HybridConfig(
    vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4, num_attention_heads=2,
    num_key_value_heads=1, head_dim=128, partial_rotary_factor=0.25, linear_key_head_dim=128,
    linear_value_head_dim=128, linear_num_key_heads=2, linear_num_value_heads=2, max_position_embeddings=4096,
)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def test_hybrid_gpu_streamed_grpo_matches_fp32_oracle():
    torch.manual_seed(0)
    ref_model = HybridForCausalLM(CFG)  # fp32 CPU oracle
    model = copy.deepcopy(ref_model).to("cuda", torch.bfloat16)
    rng = random.Random(5)
    prompt = [rng.randrange(1024) for _ in range(70)]
    trajs = []
    for tid in range(3):
        turns = []
        for _ in range(2):
            a = [rng.randrange(1024) for _ in range(rng.randint(20, 90))]
            o = [rng.randrange(1024) for _ in range(5)]
            turns.append((a + o, [True] * len(a) + [False] * len(o)))
        trajs.append((tid, turns, float(tid % 2)))
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
        got = run.logprobs(tid).float().cpu()
        want = _lp(ref_model, prompt, turns).detach()
        assert (got - want).abs().max().item() < 0.15
        bw.close_trajectory(tid, rw)
    bw.close_group(0)
    bw.assert_safe_to_step()
    bad = []
    for (n, p), (_, q) in zip(model.named_parameters(), ref_model.named_parameters()):
        e = _rel(p.grad.float().cpu(), q.grad)
        if e > 0.08:
            bad.append((n, e))
    assert not bad, bad


def test_hybrid_gpu_head_dim_256():
    """The config-5 attention geometry (head_dim 256, partial rotary) on the GPU kernels."""
    cfg = CFG.with_(head_dim=256, num_attention_heads=4, num_key_value_heads=1)
    torch.manual_seed(1)
    ref_model = HybridForCausalLM(cfg)
    model = copy.deepcopy(ref_model).to("cuda", torch.bfloat16)
    rng = random.Random(9)
    prompt = [rng.randrange(1024) for _ in range(100)]
    turns = [([rng.randrange(1024) for _ in range(150)], [True] * 150)]
    run = StreamingRun(model, boundary_cut=True)
    bw = RewardLinearBackward(run, model)
    bw.open_group(0, prompt, [0, 1])
    for tid in (0, 1):
        run.append_turn(0, tid, turns[0][0][: 150 - 40 * tid], [True] * (150 - 40 * tid))
        got = run.logprobs(tid).float().cpu()
        want = _lp(ref_model, prompt, [(turns[0][0][: 150 - 40 * tid], [True] * (150 - 40 * tid))]).detach()
        assert (got - want).abs().max().item() < 0.15
        bw.close_trajectory(tid, float(tid))
    bw.close_group(0)
    bw.assert_safe_to_step()
    assert all(p.grad is None or torch.isfinite(p.grad).all() for p in model.parameters())
