"""OPD objectives vs an independent monolithic reference (CPU fp32)."""

from __future__ import annotations

import copy
import random

import pytest
import torch

from tests.grpo_fixtures import build_model
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.opd.objectives import OPDStream, OPDTurnStream


def _episodes(seed=0, groups=2, per_group=2):
    rng = random.Random(seed)
    out = []
    tid = 0
    for g in range(groups):
        prompt = [rng.randrange(512) for _ in range(12)]
        trajs = []
        for _ in range(per_group):
            turns = []
            for k in range(rng.randint(2, 3)):
                a = [rng.randrange(512) for _ in range(rng.randint(2, 5))]
                obs = [rng.randrange(512) for _ in range(rng.randint(1, 3))]
                toks = a + obs
                sc = [True] * len(a) + [False] * len(obs)
                teacher = -torch.rand(len(a), dtype=torch.float64).float() * 3
                turns.append((toks, sc, teacher))
            trajs.append((tid, turns))
            tid += 1
        out.append((g, prompt, trajs))
    return out


def _reference(model, eps):
    model.zero_grad(set_to_none=True)
    total, mass = 0.0, 0
    for g, prompt, trajs in eps:
        for tid, turns in trajs:
            lp = reference_logprobs(model, prompt, [(tk, sc) for tk, sc, _ in turns])
            teacher = torch.cat([t for _, _, t in turns])
            total = total + ((lp.detach() - teacher) * lp).sum()
            mass += lp.numel()
    (total / mass).backward()
    return {n: p.grad.clone() for n, p in model.named_parameters()}


def test_turn_stream_matches_monolithic():
    model = build_model(5).eval()
    eps = _episodes(0)
    ref = _reference(copy.deepcopy(model), eps)
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    obj = OPDTurnStream(run, model)
    for g, prompt, _ in eps:
        obj.open_group(g, prompt)
    # interleave turns across trajectories
    queues = [(g, tid, list(turns)) for g, _, trajs in eps for tid, turns in trajs]
    while any(q[2] for q in queues):
        for g, tid, turns in queues:
            if turns:
                tk, sc, teacher = turns.pop(0)
                obj.append_scored_turn(g, tid, tk, sc, teacher_logprobs=teacher)
    for g, _, trajs in eps:
        for tid, _ in trajs:
            obj.close_trajectory(tid)
        obj.close_group(g)
    obj.assert_safe_to_step()
    for n, p in model.named_parameters():
        torch.testing.assert_close(p.grad, ref[n], rtol=2e-4, atol=2e-6, msg=n)
    assert obj.loss_value == pytest.approx(obj.loss_value)


@pytest.mark.parametrize("joint", [False, True])
def test_opd_stream_with_teacher_model(joint):
    """Per-trajectory closes, or one call closing the group's trajectories with one joint backward."""
    model = build_model(6)
    teacher = build_model(7)
    eps = _episodes(1, groups=1, per_group=3)
    # teacher scores from the teacher model (reference path)
    for g, prompt, trajs in eps:
        for i, (tid, turns) in enumerate(trajs):
            tl = reference_logprobs(teacher, prompt, [(tk, sc) for tk, sc, _ in turns]).detach()
            splits = [sum(sc) for _, sc, _ in turns]
            parts = torch.split(tl, splits)
            trajs[i] = (tid, [(tk, sc, t) for (tk, sc, _), t in zip(turns, parts)])
    ref = _reference(copy.deepcopy(model), eps)
    run = StreamingRun(model, boundary_cut=True)
    obj = OPDStream(run, model, teacher=teacher, joint_backward=joint)
    for g, prompt, trajs in eps:
        obj.open_group(g, prompt)
        for tid, turns in trajs:
            for tk, sc, _ in turns:
                run.append_turn(g, tid, tk, sc)
        if joint:
            obj.close_trajectories([tid for tid, _ in trajs])
        else:
            for tid, _ in trajs:
                obj.close_trajectory(tid)
        obj.close_group(g)
    obj.assert_safe_to_step()
    for n, p in model.named_parameters():
        torch.testing.assert_close(p.grad, ref[n], rtol=5e-4, atol=5e-6, msg=n)


def test_turn_stream_rejects_bad_inputs():
    model = build_model(0).eval()
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    obj = OPDTurnStream(run, model)
    obj.open_group(0, [1, 2, 3])
    with pytest.raises(ValueError):
        obj.append_scored_turn(0, 0, [4, 5], [True, True], teacher_logprobs=torch.tensor([-1.0]))
    with pytest.raises(ValueError):
        obj.append_scored_turn(0, 0, [4, 5], [True, True], teacher_logprobs=torch.tensor([-1.0, float("nan")]))
    with pytest.raises(RuntimeError):
        obj.assert_safe_to_step()
    with pytest.raises(ValueError):
        OPDTurnStream(StreamingRun(model, boundary_cut=True), model)


def test_turn_packs_and_closure_cohorts_match_single_turns():
    """Scored turns appended as cross-trajectory packs, and trajectories closed as one cohort, give the same
    update as one turn / one close at a time (the OPD deferred-replay invariants)."""
    model = build_model(8).eval()
    eps = _episodes(3, groups=2, per_group=2)
    res = []
    for packed in (False, True):
        m = copy.deepcopy(model)
        run = StreamingRun(m, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
        obj = OPDTurnStream(run, m)
        for g, prompt, _ in eps:
            obj.open_group(g, prompt)
        queues = [(g, tid, list(turns)) for g, _, trajs in eps for tid, turns in trajs]
        while any(q[2] for q in queues):
            items = []
            for g, tid, turns in queues:
                if turns:
                    tk, sc, teacher = turns.pop(0)
                    items.append((g, tid, tk, sc, teacher, None))
            if packed:
                obj.append_scored_turns(items)
            else:
                for g, tid, tk, sc, teacher, _ in items:
                    obj.append_scored_turn(g, tid, tk, sc, teacher_logprobs=teacher)
        for g, _, trajs in eps:
            if packed:
                obj.close_trajectories([tid for tid, _ in trajs])
            else:
                for tid, _ in trajs:
                    obj.close_trajectory(tid)
            obj.close_group(g)
        obj.assert_safe_to_step()
        res.append({n: p.grad.clone() for n, p in m.named_parameters()})
        if packed:  # the cohort's ready turns replayed as joint packs of two
            assert "2" in run.turn_path_counts["replay"], run.turn_path_counts
    for n in res[0]:
        torch.testing.assert_close(res[0][n], res[1][n], rtol=1e-5, atol=5e-6, msg=n)


def test_joint_turn_pack_rule():
    """joint_turn_pack_ready / joint_turn_replay_ready and the pack width (reference semantics: every turn
    without the checkpoint flag, none without a reserve, none when adjoints need a per-source order)."""
    model = build_model(9).eval()
    items = [(0, 0, [1, 2], [True, True]), (0, 1, [3], [True]), (0, 2, [4, 5, 6], [True, False, True])]
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    assert run.joint_turn_pack_ready and run.joint_turn_replay_ready
    assert run.joint_turn_pack_width(items) == 3
    assert run.joint_turn_pack_width(items[:1]) == 1
    assert run._turn_replay_pack([(2, 5), (1, 7)]) == [0, 1]
    ck = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True, checkpoint=True)
    assert ck.joint_turn_pack_width(items) == 1 and ck._turn_replay_pack([(2, 5), (1, 7)]) == [0]
    ck_reserve = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True,
                              checkpoint=True, rebuild_plain_reserve_bytes=0)
    assert ck_reserve.joint_turn_pack_width(items) == 3  # no device memory to read on the CPU: everything fits
    for kw in ({"parameter_adjoint_reduction": "canonical_source"}, {"explicit_adjoint_vjp": True}):
        other = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True, **kw)
        assert not other.joint_turn_pack_ready and other.joint_turn_pack_width(items) == 1
    plain = StreamingRun(model, boundary_cut=True)
    assert not plain.joint_turn_pack_ready and not plain.joint_turn_replay_ready
    assert run.shared_prefix_finalization_diagnostics() == run.shared_prefix_vjp_diagnostics()


def test_turn_stream_refuses_duplicates_and_late_turns():
    model = build_model(0).eval()
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    obj = OPDTurnStream(run, model)
    obj.open_group(0, [1, 2, 3])
    t = torch.tensor([-1.0])
    with pytest.raises(ValueError, match="twice"):
        obj.append_scored_turns([(0, 0, [4], [True], t, None), (0, 0, [5], [True], t, None)])
    with pytest.raises(ValueError):
        obj.append_scored_turns([])
    obj.append_scored_turn(0, 0, [4, 6], [True, False], teacher_logprobs=t)
    obj.close_trajectory(0)
    with pytest.raises(RuntimeError, match="closed"):
        obj.append_scored_turn(0, 0, [7], [True], teacher_logprobs=t)
    with pytest.raises(ValueError, match="twice"):
        obj.close_trajectories([1, 1])
