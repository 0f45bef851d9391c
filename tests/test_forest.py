"""Segment forest, plan and forest log-probs vs per-trajectory reference (CPU fp32)."""

from __future__ import annotations

import copy
import random

import torch

from tests.grpo_fixtures import build_model
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.plan import compile_plan, visibility_mask
from thundersync_b200.engine.segments import Segment, Trajectory, build_forest, unshared
from thundersync_b200.engine.step import forest_logprobs, split_by_trajectory


def _batch(seed=0):
    rng = random.Random(seed)
    trajs = []
    tid = 0
    for g in range(2):
        prompt = [rng.randrange(512) for _ in range(10)]
        shared_action = [rng.randrange(512) for _ in range(4)]
        for j in range(3):
            segs = [Segment.prompt(prompt)]
            if j < 2:
                segs.append(Segment.action(shared_action + [rng.randrange(512) for _ in range(3)]))
            else:
                segs.append(Segment.action([rng.randrange(512) for _ in range(5)]))
            segs.append(Segment.observation([rng.randrange(512) for _ in range(2)]))
            segs.append(Segment.action([rng.randrange(512) for _ in range(3)]))
            trajs.append(Trajectory(segs, group_id=g, traj_id=tid))
            tid += 1
    return trajs


def test_forest_is_exact_and_shares():
    trajs = _batch()
    f = build_forest(trajs)
    for t in trajs:
        path = f.path_to_root(f.leaf_of[t.traj_id])
        toks = [x for n in path for x in f.nodes[n].tokens]
        sc = [x for n in path for x in f.nodes[n].scored]
        assert toks == t.tokens and sc == t.scored_mask
    assert f.physical_tokens < f.logical_tokens
    assert build_forest(unshared(trajs)).physical_tokens == f.logical_tokens


def test_plan_mask_matches_subtree_rule():
    plan = compile_plan(build_forest(_batch()))
    m = visibility_mask(plan)
    p = plan.n_physical
    q = torch.arange(p)[:, None]
    k = torch.arange(p)[None, :]
    rule = (k <= q) & (q < plan.subtree_end[None, :])
    assert torch.equal(m, rule)


def test_forest_logprobs_match_per_trajectory_reference():
    model = build_model(3)
    trajs = _batch(1)
    plan = compile_plan(build_forest(trajs))
    lp = forest_logprobs(model, plan)
    per = split_by_trajectory(plan, lp)
    total = 0.0
    for t in trajs:
        turns = [(list(s.tokens), [s.scored] * len(s)) for s in t.segments[1:]]
        ref = reference_logprobs(model, list(t.segments[0].tokens), turns)
        torch.testing.assert_close(per[t.traj_id], ref, rtol=1e-4, atol=1e-5)
        total = total + per[t.traj_id].sum() * (t.traj_id + 1)
    total.backward()
    got = {n: p.grad.clone() for n, p in model.named_parameters()}
    model.zero_grad()
    ref_total = 0.0
    for t in trajs:
        turns = [(list(s.tokens), [s.scored] * len(s)) for s in t.segments[1:]]
        ref_total = ref_total + reference_logprobs(model, list(t.segments[0].tokens), turns).sum() * (t.traj_id + 1)
    ref_total.backward()
    for n, p in model.named_parameters():
        torch.testing.assert_close(got[n], p.grad, rtol=2e-4, atol=2e-6)


def _forest_grads(model, plan, **kw):
    model.zero_grad(set_to_none=True)
    lp = forest_logprobs(model, plan, **kw)
    (lp * torch.linspace(0.5, 1.5, lp.numel())).sum().backward()
    return lp.detach(), {n: p.grad.clone() for n, p in model.named_parameters()}


def test_checkpointed_forest_with_attention_cache_is_exact():
    """Checkpointed forest: identical log-probs and gradients; the recompute reuses kept attention outputs."""
    from thundersync_b200.ops.attention import AttentionOutputCache

    model = build_model(4)
    plan = compile_plan(build_forest(_batch(2)))
    lp0, g0 = _forest_grads(model, plan)
    for budget, expect_replay in ((1 << 30, True), (0, False)):
        cache = AttentionOutputCache(budget)
        lp1, g1 = _forest_grads(model, plan, checkpoint=True, attention_cache=cache)
        torch.testing.assert_close(lp1, lp0, rtol=0, atol=0)
        for n in g0:
            torch.testing.assert_close(g1[n], g0[n], rtol=1e-6, atol=1e-7)
        rep = cache.report()
        if expect_replay:
            assert rep["saved"] > 0 and rep["replayed"] == rep["saved"] and rep["declined"] == 0
        else:
            assert rep["saved"] == 0 and rep["declined"] > 0 and rep["replayed"] == 0


def test_forest_context_binds_and_restores_plans():
    """forest_logprobs without a plan runs the bound one; nested contexts restore the outer plan."""
    import pytest

    from thundersync_b200.engine.step import bound_plan, forest_context

    model = build_model(5)
    outer = compile_plan(build_forest(_batch(3)))
    inner = compile_plan(build_forest(_batch(4)))
    assert bound_plan("cpu") is None
    with pytest.raises(RuntimeError):
        forest_logprobs(model)
    with forest_context(outer):
        lp_outer = forest_logprobs(model)
        with forest_context(inner):
            assert bound_plan("cpu") is inner
            torch.testing.assert_close(forest_logprobs(model), forest_logprobs(model, inner), rtol=0, atol=0)
        assert bound_plan("cpu") is outer
        lp_outer.sum().backward()  # the step's backward inside the context, as with checkpointing
    assert bound_plan("cpu") is None
    torch.testing.assert_close(lp_outer.detach(), forest_logprobs(model, outer).detach(), rtol=0, atol=0)


def test_every_share_and_gate_setting_is_the_same_computation():
    """Shared or unshared forest, gated head or every position projected: same log-probs and gradients."""
    base = build_model(6)
    trajs = _batch(5)
    res = []
    for share in (True, False):
        for gate in (True, False):
            m = copy.deepcopy(base)
            forest = build_forest(trajs if share else unshared(trajs))
            plan = compile_plan(forest)
            lp = forest_logprobs(m, plan, gate=gate)
            (lp * torch.linspace(0.5, 1.5, lp.numel())).sum().backward()
            res.append((lp.detach(), {n: p.grad for n, p in m.named_parameters()}, plan))
    lp0, g0, p0 = res[0]
    for lp, g, plan in res[1:]:
        torch.testing.assert_close(lp, lp0, rtol=1e-5, atol=1e-6)
        for n in g0:  # fp32 summation order differs: compare in norm
            assert float((g[n] - g0[n]).norm() / g0[n].norm().clamp_min(1e-30)) < 1e-5, n
    shared_plan, unshared_plan = res[0][2], res[2][2]
    assert shared_plan.n_physical < unshared_plan.n_physical  # the shared forest forwards fewer tokens
    assert unshared_plan.n_physical == shared_plan.forest.logical_tokens  # unshared shares nothing


def test_the_executor_cache_does_not_keep_a_dropped_model_alive():
    import gc
    import weakref

    m = build_model(7)
    plan = compile_plan(build_forest(_batch(6)))
    forest_logprobs(m, plan).sum().backward()
    ref = weakref.ref(m)
    del m
    gc.collect()
    assert ref() is None
