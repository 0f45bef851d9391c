"""On-policy distillation turn streams defer turns without a scored token.

Such a turn has no loss; its K/V and last hidden state are read only by later turns of its trajectory.
It forwards when the trajectory's next turn arrives (as its own single-turn call at its own positions),
and a trailing one is never forwarded. The losses and gradients equal the forward-at-arrival run
exactly (behaviour of reference tests/opd/test_opd_deferred_unscored_turns.py:87-130; CPU fp32).
"""

from __future__ import annotations

import copy

import torch

from tests.grpo_fixtures import build_model
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.opd.objectives import OPDTurnStream

# unscored opener, action, unscored middle, action, trailing unscored observation
TURNS = [([3, 4], [False, False]), ([5, 6, 7], [False, True, True]), ([8, 9, 10, 11], [False] * 4),
         ([12, 13], [True, True]), ([14, 15, 16], [False] * 3)]


def _teacher(n, seed):
    g = torch.Generator().manual_seed(seed)
    return -torch.rand(n, generator=g) * 3


def _run(model, defer: bool, trajs=(0, 1)):
    run = StreamingRun(model, boundary_cut=True, stream_turns=True, turn_boundary_rebuild=True)
    obj = OPDTurnStream(run, model)
    run.defer_unscored_turns = defer
    obj.open_group(0, [1, 2])
    losses = []
    for k, (tk, sc) in enumerate(TURNS):  # turns of both trajectories arrive round-robin
        for tid in trajs:
            losses.append(obj.append_scored_turn(0, tid, tk, sc, teacher_logprobs=_teacher(sum(sc), 10 * k + tid)))
    counts = (run._counts["turn_forward"], run._deferred_turns, run._deferred_forwards)
    obj.close_trajectories(list(trajs))
    obj.close_group(0)
    obj.assert_safe_to_step()
    return losses, {n: p.grad.detach().clone() for n, p in model.named_parameters()}, counts, run


def test_deferral_preserves_losses_and_gradients_exactly():
    base = build_model(81).eval()
    la, ga, _, _ = _run(copy.deepcopy(base), defer=False)
    lb, gb, _, _ = _run(copy.deepcopy(base), defer=True)
    assert la == lb
    for n in ga:
        assert torch.equal(ga[n], gb[n]), n


def test_only_the_trailing_unscored_turn_is_left_unforwarded():
    _, _, (forwards, deferred, caught_up), _ = _run(build_model(82).eval(), defer=True)
    # per trajectory: 5 turns, 3 unscored (opener, middle, trailing); the opener and the middle forward
    # when the next action arrives, the trailing one never
    assert deferred == 2 * 3 and caught_up == 2 * 2 and forwards == 2 * 4


def test_a_closed_trajectory_holds_no_deferred_turn():
    _, _, _, run = _run(build_model(83).eval(), defer=True, trajs=(0,))
    assert 0 not in run._trajs
