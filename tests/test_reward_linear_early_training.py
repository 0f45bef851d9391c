"""Early training: sources computed before their rewards (prepare), folded when the reward arrives (bind).

CPU fp32 on the config-1 tiny model. The behaviours are the ones the reference's early-training battery
checks (reference tests/test_reward_linear_early_training.py:122-342), stated against this package's
API: binding order does not change the gradient beyond fp32 summation order; a reward may also arrive
before its trajectory's content (the known-reward path); duplicate prepares, conflicting rewards,
non-finite rewards, early group closes and parameter updates inside the batch are refused; abort frees
held sources.
"""

from __future__ import annotations

import copy

import pytest
import torch

from tests.grpo_fixtures import EPS, build_model, make_batch
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _setup(model):
    run = StreamingRun(model, boundary_cut=True, stream_turns=False)
    return run, RewardLinearBackward(run, model, eps=EPS)


def _append(run, g, turns, tid):
    for tk, sc in turns:
        run.append_turn(g, tid, tk, sc)


def _grads(model):
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


def _run(model, batch, drive):
    m = copy.deepcopy(model)
    run, bw = _setup(m)
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    drive(run, bw)
    for g, _, _ in batch:
        bw.close_group(g)
    bw.assert_safe_to_step()
    return _grads(m)


def _close_path(batch):
    def drive(run, bw):
        for g, _, trajs in batch:
            for tid, turns, reward in trajs:
                _append(run, g, turns, tid)
                bw.close_trajectory(tid, reward)
    return drive


def _assert_same(a, b):
    for n in a:
        torch.testing.assert_close(a[n], b[n], rtol=1e-5, atol=1e-6, msg=n)


def test_binding_in_reverse_order_equals_the_close_path():
    model = build_model(21)
    batch, _ = make_batch(21, groups=2, per_group=4)

    def drive(run, bw):
        for g, _, trajs in batch:
            for tid, turns, _ in trajs:
                _append(run, g, turns, tid)
                bw.prepare_trajectory(tid)
        assert bw.held_source_count == sum(len(t) for _, _, t in batch)
        binds = [(tid, reward) for _, _, trajs in batch for tid, _, reward in trajs]
        for tid, reward in reversed(binds):
            bw.bind_reward(tid, reward)
        assert bw.held_source_count == 0

    _assert_same(_run(model, batch, drive), _run(model, batch, _close_path(batch)))


def test_reward_before_content_takes_the_known_reward_path():
    """A reward recorded before the trajectory is prepared is differentiated at prepare time."""
    model = build_model(22)
    batch, _ = make_batch(22, groups=1, per_group=4)

    def drive(run, bw):
        for g, _, trajs in batch:
            bw.record_rewards([(tid, reward) for tid, _, reward in trajs])
            for tid, turns, _ in trajs:
                _append(run, g, turns, tid)
                bw.prepare_trajectory(tid)
            assert bw.held_source_count == 0  # nothing waits for a reward

    _assert_same(_run(model, batch, drive), _run(model, batch, _close_path(batch)))


def test_a_group_with_every_source_prepared_is_not_bound_until_the_rewards_arrive():
    model = build_model(23)
    batch, _ = make_batch(23, groups=1, per_group=3)
    run, bw = _setup(model)
    g, prompt, trajs = batch[0]
    bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for tid, turns, _ in trajs:
        _append(run, g, turns, tid)
        bw.prepare_trajectory(tid)
    assert not bw.group_fully_bound(g)
    for tid, _, reward in trajs[:-1]:
        bw.bind_reward(tid, reward)
    with pytest.raises(RuntimeError):
        bw.close_group(g)  # the straggler still holds its group open
    with pytest.raises(RuntimeError):
        bw.assert_safe_to_step()
    tid, _, reward = trajs[-1]
    bw.bind_reward(tid, reward)
    assert bw.group_fully_bound(g)
    bw.close_group(g)
    bw.assert_safe_to_step()


def test_duplicate_prepare_conflicting_or_non_finite_rewards_are_refused():
    model = build_model(24)
    batch, _ = make_batch(24, groups=1, per_group=2)
    run, bw = _setup(model)
    g, prompt, trajs = batch[0]
    bw.open_group(g, prompt, [t for t, _, _ in trajs])
    (t0, turns0, _), (t1, turns1, _) = trajs
    _append(run, g, turns0, t0)
    bw.prepare_trajectory(t0)
    with pytest.raises(ValueError):
        bw.prepare_trajectory(t0)
    with pytest.raises(ValueError):
        bw.bind_reward(t0, float("nan"))
    with pytest.raises(ValueError):
        bw.bind_reward(t0, float("inf"))
    bw.record_rewards([(t1, 1.0)])
    with pytest.raises(ValueError):
        bw.record_rewards([(t1, 0.0)])
    bw.record_rewards([(t1, 1.0)])  # the same reward again is not a conflict
    with pytest.raises(KeyError):
        bw.prepare_trajectory(10_000)  # not registered with any group


def test_a_parameter_update_between_prepare_and_bind_is_refused():
    model = build_model(25)
    batch, _ = make_batch(25, groups=1, per_group=2)
    run, bw = _setup(model)
    g, prompt, trajs = batch[0]
    bw.open_group(g, prompt, [t for t, _, _ in trajs])
    (t0, turns0, _), (t1, turns1, _) = trajs
    _append(run, g, turns0, t0)
    bw.prepare_trajectory(t0)
    with torch.no_grad():
        next(model.parameters()).add_(1e-3)  # an optimizer step inside the logical batch
    _append(run, g, turns1, t1)
    with pytest.raises(RuntimeError, match="version guard"):
        bw.prepare_trajectory(t1)


def test_abort_frees_held_sources_and_refuses_the_step():
    model = build_model(26)
    batch, _ = make_batch(26, groups=2, per_group=2)
    run, bw = _setup(model)
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    g, _, trajs = batch[0]
    for tid, turns, _ in trajs:
        _append(run, g, turns, tid)
        bw.prepare_trajectory(tid)
    assert bw.held_source_count == 2 and bw.retained_device_bytes()["held_sources"] > 0
    bw.abort()
    assert bw.held_source_count == 0 and bw.retained_device_bytes()["held_sources"] == 0
    assert bw.open_groups() == []
    with pytest.raises(RuntimeError):
        bw.assert_safe_to_step()


def test_deferred_group_closes_run_in_request_order_at_later_safe_points(monkeypatch):
    """defer_group_close: a close that would wait for host folds returns at once and runs later, in
    request order; the gradient equals closing at once bitwise."""
    model = build_model(27)
    batch, _ = make_batch(27, groups=3, per_group=2)
    ref = _run(model, batch, _close_path(batch))

    m = copy.deepcopy(model)
    run = StreamingRun(m, boundary_cut=True, stream_turns=False)
    bw = RewardLinearBackward(run, m, eps=EPS, defer_group_close=True)
    pending = {"on": True}
    monkeypatch.setattr(bw, "_folds_pending", lambda: pending["on"])
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    order = []
    real = bw._close_group_now
    monkeypatch.setattr(bw, "_close_group_now", lambda g: (order.append(g), real(g)))
    (g0, _, t0), (g1, _, t1), (g2, _, t2) = batch
    for g, trajs in ((g0, t0), (g1, t1)):
        for tid, turns, reward in trajs:
            _append(run, g, turns, tid)
            bw.close_trajectory(tid, reward)
        bw.close_group(g)
    assert order == [] and bw.open_groups() == [g0, g1, g2]
    assert bw.source_offload_report["group_closes_deferred"] == 2
    with pytest.raises(RuntimeError):
        bw.close_group(g0)  # already requested
    pending["on"] = False
    tid, turns, reward = t2[0]
    _append(run, g2, turns, tid)
    bw.close_trajectory(tid, reward)  # a safe point: both requested closes run, in order
    assert order == [g0, g1] and bw.open_groups() == [g2]
    tid, turns, reward = t2[1]
    _append(run, g2, turns, tid)
    bw.close_trajectory(tid, reward)
    pending["on"] = True
    bw.close_group(g2)
    assert order == [g0, g1]
    bw.assert_safe_to_step()  # waits, then runs the last request
    assert order == [g0, g1, g2]
    got = {n: p.grad.detach().clone() for n, p in m.named_parameters()}
    for n in ref:
        assert torch.equal(got[n], ref[n]), n


def test_reduction_hooks_follow_the_host_fold_pipeline():
    """group_reduction_complete / pending_reduction_source_count / wait_for_trajectory_reduction read the
    host fold pipeline (a stand-in here: the real one streams from a CUDA device)."""

    class FakePipe:
        def __init__(self):
            self.running = 2
            self.drains = 0

        def pending_count(self):
            return self.running

        def pending(self):
            return self.running > 0

        def drain(self):
            self.drains += 1
            self.running = 0

    model = build_model(28)
    batch, _ = make_batch(28, groups=1, per_group=2)
    run, bw = _setup(model)
    g, prompt, trajs = batch[0]
    bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for tid, turns, reward in trajs:
        _append(run, g, turns, tid)
        bw.close_trajectory(tid, reward)
    assert bw.group_reduction_complete(g) and bw.pending_reduction_source_count == 0
    pipe = FakePipe()
    bw._host_fold = pipe
    assert not bw.group_reduction_complete(g) and bw.pending_reduction_source_count == 2
    with pytest.raises(KeyError):
        bw.wait_for_trajectory_reduction(g, 10_000)
    bw.wait_for_trajectory_reduction(g, trajs[0][0])
    assert pipe.drains == 1 and bw.group_reduction_complete(g)
    bw._host_fold = None
    bw.close_group(g)
    bw.assert_safe_to_step()
