"""Config 1: streamed GRPO gradient == non-streaming full-batch reference (CPU fp32)."""

from __future__ import annotations

import copy

import pytest
import torch

from tests.grpo_fixtures import EPS, advantages, build_model, make_batch
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _reference_grads(model, batch):
    model.zero_grad(set_to_none=True)
    total = 0.0
    for g, prompt, trajs in batch:
        adv = advantages([r for _, _, r in trajs])
        for (tid, turns, _), a in zip(trajs, adv):
            lp = reference_logprobs(model, prompt, turns)
            total = total + a * lp.sum()
    total.backward()
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


def _streamed_grads(model, batch, order, *, stream_turns, binary=False, mode="blocking", direct=False):
    model.zero_grad(set_to_none=True)
    run = StreamingRun(model, boundary_cut=True, stream_turns=stream_turns)
    bw = RewardLinearBackward(run, model, eps=EPS, source_offload_mode=mode, direct_when_group_bound=direct)
    if binary:
        bw.configure_binary_rewards()
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    if direct:
        for g, _, trajs in batch:
            bw.record_rewards([(t, r) for t, _, r in trajs])
    for g, (tid, turns, reward) in order:
        for tk, sc in turns:
            run.append_turn(g, tid, tk, sc)
        bw.close_trajectory(tid, reward)
    for g, _, _ in batch:
        bw.close_group(g)
    bw.assert_safe_to_step()
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


@pytest.mark.parametrize("stream_turns", [True, False])
@pytest.mark.parametrize("binary", [False, True])
def test_streamed_equals_full_batch(stream_turns, binary):
    model = build_model(0)
    batch, order = make_batch(0)
    ref = _reference_grads(copy.deepcopy(model), batch)
    got = _streamed_grads(model, batch, order, stream_turns=stream_turns, binary=binary)
    for name, g in ref.items():
        torch.testing.assert_close(got[name], g, rtol=2e-4, atol=2e-6, msg=name)


def test_multi_turn_with_unscored_observations():
    model = build_model(1)
    batch, order = make_batch(1, multi_turn=True)
    ref = _reference_grads(copy.deepcopy(model), batch)
    got = _streamed_grads(model, batch, order, stream_turns=True)
    for name, g in ref.items():
        torch.testing.assert_close(got[name], g, rtol=2e-4, atol=2e-6, msg=name)


def test_direct_when_group_bound_matches():
    model = build_model(2)
    batch, order = make_batch(2)
    ref = _reference_grads(copy.deepcopy(model), batch)
    got = _streamed_grads(model, batch, order, stream_turns=False, direct=True)
    for name, g in ref.items():
        torch.testing.assert_close(got[name], g, rtol=2e-4, atol=2e-6, msg=name)


def test_step_with_open_group_raises():
    model = build_model(0)
    run = StreamingRun(model, boundary_cut=True)
    bw = RewardLinearBackward(run, model)
    bw.open_group(0, [1, 2, 3], [0, 1])
    run.append_turn(0, 0, [4, 5], [True, True])
    bw.close_trajectory(0, 1.0)
    with pytest.raises(RuntimeError, match="still open"):
        bw.assert_safe_to_step()


def test_version_guard_fires():
    model = build_model(0)
    run = StreamingRun(model, boundary_cut=True)
    bw = RewardLinearBackward(run, model)
    bw.open_group(0, [1, 2, 3], [0, 1])
    run.append_turn(0, 0, [4, 5], [True, True])
    with torch.no_grad():
        next(model.parameters()).add_(1.0)
    with pytest.raises(RuntimeError, match="version guard|changed inside"):
        bw.close_trajectory(0, 1.0)


@pytest.mark.parametrize("binary", [False, True])
def test_uniform_reward_group(binary):
    """A group whose rewards are all equal contributes A*G2 (A exactly 0 here)."""
    model = build_model(4)
    batch, order = make_batch(4)
    batch = [(g, p, [(t, turns, 1.0 if g == 0 else r) for t, turns, r in trajs]) for g, p, trajs in batch]
    rewards = {t: r for _, _, trajs in batch for t, _, r in trajs}
    order = [(g, (t, turns, rewards[t])) for g, (t, turns, _) in order]
    ref = _reference_grads(copy.deepcopy(model), batch)
    got = _streamed_grads(model, batch, order, stream_turns=False, binary=binary)
    for name, g in ref.items():
        torch.testing.assert_close(got[name], g, rtol=2e-4, atol=2e-6, msg=name)
