"""Reward-linear GRPO objective invariants (CPU fp32; the reference's reward-linear test battery, restated).

- prepare + bind == close (bitwise);
- the binary-reward statistic path equals the general one;
- source placement (blocking / device-resident) does not change the gradient;
- a group is closed only when every trajectory is bound, and stepping with an open group fails loudly;
- abort frees every open group; retained memory is reported per kind.
"""

from __future__ import annotations

import copy

import pytest
import torch

from tests.grpo_fixtures import EPS, build_model, make_batch
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _setup(model, *, binary=False, **bw_kw):
    run = StreamingRun(model, boundary_cut=True, stream_turns=False)
    bw = RewardLinearBackward(run, model, eps=EPS, **bw_kw)
    if binary:
        bw.configure_binary_rewards()
    return run, bw


def _grads(model):
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


def _append(run, g, turns, tid):
    for tk, sc in turns:
        run.append_turn(g, tid, tk, sc)


def test_prepare_then_bind_equals_close():
    model = build_model(11)
    batch, order = make_batch(11)
    res = []
    for split in (False, True):
        m = copy.deepcopy(model)
        run, bw = _setup(m)
        for g, prompt, trajs in batch:
            bw.open_group(g, prompt, [t for t, _, _ in trajs])
        for g, (tid, turns, reward) in order:
            _append(run, g, turns, tid)
            if split:
                bw.prepare_trajectory(tid)
                bw.bind_reward(tid, reward)
            else:
                bw.close_trajectory(tid, reward)
        for g, _, _ in batch:
            bw.close_group(g)
        bw.assert_safe_to_step()
        res.append(_grads(m))
    for n in res[0]:
        assert torch.equal(res[0][n], res[1][n]), n


def test_binary_statistics_equal_general_path():
    model = build_model(12)
    batch, order = make_batch(12)
    res = []
    for binary in (False, True):
        m = copy.deepcopy(model)
        run, bw = _setup(m, binary=binary)
        for g, prompt, trajs in batch:
            bw.open_group(g, prompt, [t for t, _, _ in trajs])
        for g, (tid, turns, reward) in order:
            _append(run, g, turns, tid)
            bw.close_trajectory(tid, reward)
        for g, _, _ in batch:
            bw.close_group(g)
        bw.assert_safe_to_step()
        res.append(_grads(m))
    for n in res[0]:
        torch.testing.assert_close(res[0][n], res[1][n], rtol=1e-5, atol=5e-6, msg=n)


def test_group_closes_only_when_bound_and_open_step_fails():
    model = build_model(13)
    batch, order = make_batch(13, groups=1, per_group=3)
    run, bw = _setup(model)
    g, prompt, trajs = batch[0]
    bw.open_group(g, prompt, [t for t, _, _ in trajs])
    assert g in bw.open_groups() and not bw.group_fully_bound(g)
    (tid, turns, reward) = trajs[0]
    _append(run, g, turns, tid)
    bw.close_trajectory(tid, reward)
    with pytest.raises(RuntimeError):
        bw.assert_safe_to_step()
    for tid, turns, reward in trajs[1:]:
        _append(run, g, turns, tid)
        bw.close_trajectory(tid, reward)
    assert bw.group_fully_bound(g)
    bw.close_group(g)
    assert g not in bw.open_groups()
    bw.assert_safe_to_step()


def test_abort_releases_open_groups_and_reports_memory():
    model = build_model(14)
    batch, order = make_batch(14)
    run, bw = _setup(model, source_offload_mode="device_resident", source_offload_device=None)
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    g, (tid, turns, reward) = order[0]
    _append(run, g, turns, tid)
    bw.close_trajectory(tid, reward)
    mem = bw.retained_device_bytes()
    assert isinstance(mem, dict) and all(isinstance(v, int) and v >= 0 for v in mem.values())
    bw.abort()
    assert bw.open_groups() == []


def test_uniform_reward_group_contributes_no_gradient():
    """All-equal rewards give zero advantages: the group adds nothing (population std normalisation)."""
    model = build_model(15)
    batch, order = make_batch(15, groups=1, per_group=4)
    g, prompt, trajs = batch[0]
    run, bw = _setup(model)
    bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for tid, turns, _ in trajs:
        _append(run, g, turns, tid)
        bw.close_trajectory(tid, 1.0)
    bw.close_group(g)
    bw.assert_safe_to_step()
    for n, p in model.named_parameters():
        assert p.grad is None or float(p.grad.abs().max()) == 0.0, n
