"""The streamed execution is the monolithic execution, reordered (CPU fp32, config-1 tiny model).

Stated after reference tests/test_forest_streaming.py:128-260: gradients (not only values) match the
independent plain-torch oracle, including a loss on the last turn alone, which reaches the parameters
only through the earlier turns' K/V; the streamed log-probs equal the batch forest trainer's; old and
new log-probs are the same tensors; a group's prompt is forwarded once; a trajectory cannot change
groups; turn-boundary replay needs eval mode; HF gradient checkpointing is refused.
"""

from __future__ import annotations

import copy
import random

import pytest
import torch

from tests.grpo_fixtures import build_model
from tests.reference_model import reference_logprobs
from thundersync_b200.engine.plan import compile_plan
from thundersync_b200.engine.segments import Segment, Trajectory, build_forest
from thundersync_b200.engine.step import forest_logprobs, split_by_trajectory
from thundersync_b200.engine.streaming import StreamingRun


def _episode(seed, groups=2, per_group=2, vocab=512):
    rng = random.Random(seed)
    prompts, trajs = {}, {}
    tid = 0
    for g in range(groups):
        prompts[g] = [rng.randrange(vocab) for _ in range(rng.randint(5, 9))]
        for _ in range(per_group):
            turns = []
            for k in range(rng.randint(2, 4)):
                n = rng.randint(2, 6)
                turns.append(([rng.randrange(vocab) for _ in range(n)], [k % 2 == 0] * n))
            trajs[tid] = (g, turns)
            tid += 1
    return prompts, trajs


def _stream(model, prompts, trajs, **kw):
    run = StreamingRun(model, **kw)
    for g, p in prompts.items():
        run.open_group(g, p)
    depth = max(len(t[1]) for t in trajs.values())
    for k in range(depth):  # round-robin arrivals across trajectories and groups
        for tid, (g, turns) in trajs.items():
            if k < len(turns):
                run.append_turn(g, tid, *turns[k])
    return run


def test_a_last_turn_loss_reaches_the_parameters_through_earlier_turns():
    base = build_model(71)
    prompts, trajs = _episode(71, groups=1, per_group=1)
    sm, om = copy.deepcopy(base), copy.deepcopy(base)
    run = _stream(sm, prompts, trajs)
    tid = 0
    g, turns = trajs[tid]
    run.logprobs(tid)[-1].backward()
    reference_logprobs(om, prompts[g], turns)[-1].backward()
    for (n, p), (_, q) in zip(sm.named_parameters(), om.named_parameters()):
        if q.grad is None:
            continue
        torch.testing.assert_close(p.grad, q.grad, rtol=2e-3, atol=2e-5, msg=n)


def test_streamed_equals_the_forest_trainer_and_old_is_new_by_identity():
    base = build_model(72)
    prompts, trajs = _episode(72)
    sm, fm = copy.deepcopy(base), copy.deepcopy(base)
    run = _stream(sm, prompts, trajs)
    forest_trajs = [Trajectory([Segment.prompt(prompts[g])] + [
        Segment.action(tk) if sc[0] else Segment.observation(tk) for tk, sc in turns], group_id=g, traj_id=tid)
        for tid, (g, turns) in trajs.items()]
    plan = compile_plan(build_forest(forest_trajs))
    mono = split_by_trajectory(plan, forest_logprobs(fm, plan))
    for tid in trajs:
        torch.testing.assert_close(run.logprobs(tid), mono[tid], rtol=1e-4, atol=1e-5)
        assert torch.equal(run.logprobs(tid).detach(), run.old_logprobs(tid))


def test_the_prompt_is_forwarded_once_per_group():
    prompts, trajs = _episode(73, groups=1, per_group=4)
    run = _stream(build_model(73), prompts, trajs)
    assert run._counts["prompt_forward"] == 1


def test_a_trajectory_cannot_change_groups():
    run = StreamingRun(build_model(74))
    run.open_group(0, [1, 2, 3])
    run.open_group(1, [4, 5, 6])
    run.append_turn(0, 17, [7, 8], [True, False])
    with pytest.raises(ValueError, match="belongs to group 0"):
        run.append_turn(1, 17, [9, 10], [True, False])


def test_turn_boundary_replay_needs_eval_mode_and_hf_checkpointing_is_refused():
    model = build_model(75).train()
    with pytest.raises(ValueError, match="eval"):
        StreamingRun(model, boundary_cut=True, turn_boundary_rebuild=True)
    model.eval()
    object.__setattr__(model, "is_gradient_checkpointing", True)
    with pytest.raises(NotImplementedError, match="checkpoint"):
        StreamingRun(model)
