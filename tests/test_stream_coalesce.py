"""Coalesced turn arrivals: the turns of one scheduling window handed over in one call.

``StreamingRun.append_turns`` records the turns that arrived in one window. With
``joint_backward=True`` (the caller backwards their losses together) they forward as one pack, each
segment attending to its own trajectory's ancestor chain; otherwise each trajectory's turn forwards on
its own, so per-trajectory backwards (the reward-linear objective's) never meet a shared pack graph.
Either way coalescing changes the kernel schedule and nothing else: log-probs and parameter gradients
equal the per-turn sequential path and the independent plain-torch oracle, and the saved old
log-probs equal the new ones bitwise. Same invariant as reference
tests/test_stream_coalesce.py:130-230; here a trajectory that appears twice in one window forwards in
rounds instead of being refused, and a call with a bad item changes nothing.

CPU fp32, config-1 tiny model: 2 groups x 3 trajectories with different turn counts and lengths,
arriving round-robin so every window mixes groups, trajectories and segment lengths.
"""

from __future__ import annotations

import copy
import random

import pytest
import torch

from tests.grpo_fixtures import EPS, build_model
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _workload(seed=5, vocab=512):
    rng = random.Random(seed)
    groups, trajs = {}, {}
    tid = 0
    for g in range(2):
        groups[g] = [rng.randrange(vocab) for _ in range(rng.randint(6, 12))]
        for j in range(3):
            turns = []
            for k in range(2 + j):
                n = rng.randint(2, 9)
                scored = k % 2 == 0
                turns.append(([rng.randrange(vocab) for _ in range(n)], [scored] * n))
            trajs[tid] = (g, turns, float(rng.random() < 0.5))
            tid += 1
    windows = []
    depth = max(len(t[1]) for t in trajs.values())
    for k in range(depth):
        w = [(g, tid, turns[k][0], turns[k][1]) for tid, (g, turns, _) in trajs.items() if k < len(turns)]
        windows.append(w)
    return groups, trajs, windows


def _total(lps):
    return sum((i + 1) * lp.sum() for i, lp in sorted(lps.items()))


def _grads(model):
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


def _assert_grads(a, b, msg):
    for n in a:
        torch.testing.assert_close(a[n], b[n], rtol=2e-4, atol=2e-6, msg=lambda m, n=n: f"{msg} {n}: {m}")


@pytest.mark.parametrize("joint", [False, True])
@pytest.mark.parametrize("checkpoint", [False, True])
def test_coalesced_equals_sequential_and_oracle(checkpoint, joint):
    base = build_model(31)
    groups, trajs, windows = _workload()
    assert len(windows) >= 3 and len(windows[0]) == 6
    assert all(len({g for g, *_ in w}) == 2 for w in windows[:2])
    assert len({len(tk) for _, _, tk, _ in windows[0]}) > 1

    cm, sm, om = (copy.deepcopy(base) for _ in range(3))
    coal = StreamingRun(cm, checkpoint=checkpoint)
    seq = StreamingRun(sm, checkpoint=checkpoint)
    for run in (coal, seq):
        for g, prompt in groups.items():
            run.open_group(g, prompt)
    for w in windows:
        coal.append_turns(w, joint_backward=joint)
        for g, tid, tk, sc in w:
            seq.append_turn(g, tid, tk, sc)
    packs = coal._turn_counts["forward"]
    assert (packs.get("6", 0) >= 1) if joint else (set(packs) == {"1"})

    got = {tid: coal.logprobs(tid) for tid in trajs}
    ref = {tid: seq.logprobs(tid) for tid in trajs}
    want = {tid: reference_logprobs(om, groups[g], turns) for tid, (g, turns, _) in trajs.items()}
    for tid in trajs:
        torch.testing.assert_close(got[tid], ref[tid], rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(got[tid], want[tid], rtol=1e-4, atol=1e-5)
        assert torch.equal(got[tid].detach(), coal.old_logprobs(tid))
    _total(got).backward()
    _total(ref).backward()
    _total(want).backward()
    _assert_grads(_grads(cm), _grads(sm), "coalesced vs sequential")
    _assert_grads(_grads(cm), _grads(om), "coalesced vs oracle")


def test_a_trajectory_twice_in_one_window_forwards_in_rounds():
    base = build_model(32)
    groups = {0: [1, 2, 3, 4, 5]}
    items = [(0, 7, [7, 8, 9], [True] * 3), (0, 8, [4, 4], [True, False]), (0, 7, [10, 11], [True, True])]
    am, bm = copy.deepcopy(base), copy.deepcopy(base)
    a, b = StreamingRun(am), StreamingRun(bm)
    for run in (a, b):
        run.open_group(0, groups[0])
    a.append_turns(items)
    for g, tid, tk, sc in items:
        b.append_turn(g, tid, tk, sc)
    for tid in (7, 8):
        torch.testing.assert_close(a.logprobs(tid), b.logprobs(tid), rtol=1e-5, atol=1e-6)
    assert a.logprobs(7).numel() == 5 and a.logprobs(8).numel() == 1


def test_malformed_turns_are_refused():
    run = StreamingRun(build_model(33))
    run.open_group(0, [1, 2, 3])
    with pytest.raises(ValueError):
        run.append_turns([(0, 1, [4, 5], [True])])
    with pytest.raises(ValueError):
        run.append_turns([(0, 1, [], [])])


def test_reward_linear_over_coalesced_arrivals_equals_per_turn_arrivals():
    """Per-trajectory backwards over coalesced arrivals (each trajectory's turn forwarded on its own)."""
    base = build_model(34)
    groups, trajs, windows = _workload(seed=9)
    res = []
    for coalesce in (True, False):
        m = copy.deepcopy(base)
        run = StreamingRun(m, boundary_cut=True)
        bw = RewardLinearBackward(run, m, eps=EPS)
        for g, prompt in groups.items():
            bw.open_group(g, prompt, [tid for tid, t in trajs.items() if t[0] == g])
        for w in windows:
            if coalesce:
                run.append_turns(w)
            else:
                for g, tid, tk, sc in w:
                    run.append_turn(g, tid, tk, sc)
            for _, tid, _, _ in w:
                if len(trajs[tid][1]) == sum(1 for ww in windows[: windows.index(w) + 1]
                                             for _, t2, _, _ in ww if t2 == tid):
                    bw.close_trajectory(tid, trajs[tid][2])
        for g in groups:
            bw.close_group(g)
        bw.assert_safe_to_step()
        res.append(_grads(m))
    _assert_grads(res[0], res[1], "coalesced vs per-turn")


def test_a_bad_item_leaves_the_run_unchanged():
    run = StreamingRun(build_model(35))
    run.open_group(0, [1, 2, 3])
    with pytest.raises(KeyError):
        run.append_turns([(0, 1, [4, 5], [True, True]), (9, 2, [6], [True])])  # group 9 is not open
    with pytest.raises(ValueError):
        run.append_turns([(0, 1, [4, 5], [True, True]), (0, 2, [6], [True, False])])
    assert 1 not in run._trajs and 2 not in run._trajs
