"""Shared prompt prefixes (a radix prompt forest): when and how each shared node's one backward runs.

``open_groups_shared_prefix`` forwards every shared prefix once and cuts it like a prompt; its backward
takes the summed adjoints of every group under it. By default all shared nodes run at the batch barrier
(``assert_safe_to_step``), one autograd call per node (``"sequential"``) or per frontier of nodes whose
children are done (``"ready_frontier"``). ``dependency_ready_shared_prefix_vjp=True`` runs a node as soon
as every group under it has run its prompt backward and its shared children are done. None of these
changes the gradient beyond fp32 summation order (reference src/thundersync/engine/streaming.py:3060-3075).

CPU fp32, config-1 tiny model, reward-linear GRPO over four groups whose prompts share a two-level prefix.
"""

from __future__ import annotations

import copy
import random

import pytest
import torch

from tests.grpo_fixtures import EPS, build_model
from thundersync_b200.config import ConfigError
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _workload(seed=3, vocab=512):
    rng = random.Random(seed)
    root = [rng.randrange(vocab) for _ in range(10)]
    mid_a = [rng.randrange(vocab) for _ in range(5)]
    mid_b = [rng.randrange(vocab) for _ in range(4)]
    prompts = {
        0: root + mid_a + [rng.randrange(vocab) for _ in range(3)],
        1: root + mid_a + [rng.randrange(vocab) for _ in range(2)],
        2: root + mid_b + [rng.randrange(vocab) for _ in range(4)],
        3: root + mid_b + [rng.randrange(vocab) for _ in range(1)],
    }
    trajs = {}
    tid = 0
    for g in prompts:
        for _ in range(3):
            n = rng.randint(3, 8)
            trajs[tid] = (g, [rng.randrange(vocab) for _ in range(n)], float(rng.random() < 0.5))
            tid += 1
    return prompts, trajs


def _run(model, **run_kw):
    prompts, trajs = _workload()
    run = StreamingRun(model, boundary_cut=True, **run_kw)
    bw = RewardLinearBackward(run, model, eps=EPS)
    run.open_groups_shared_prefix(prompts)
    for g in prompts:
        bw.register_group_trajectories(g, [t for t, v in trajs.items() if v[0] == g])
    early = []
    for g in (0, 1, 2, 3):  # groups close one subtree at a time
        for t, (gg, toks, r) in trajs.items():
            if gg == g:
                run.append_turn(g, t, toks, [True] * len(toks))
                bw.close_trajectory(t, r)
        bw.close_group(g)
        early.append(run.shared_prefix_vjp_diagnostics()["finalized"])
    bw.assert_safe_to_step()
    diag = run.shared_prefix_vjp_diagnostics()
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}, early, diag


def test_the_forest_has_a_root_and_two_children():
    run = StreamingRun(build_model(1), boundary_cut=True)
    run.open_groups_shared_prefix(_workload()[0])
    assert len(run._shared) == 3
    root = [n for n in run._shared if n.parent is None]
    assert len(root) == 1 and sorted(root[0].groups) == [0, 1, 2, 3] and len(root[0].children) == 2


@pytest.mark.parametrize("kw", [{"dependency_ready_shared_prefix_vjp": True},
                                {"shared_prefix_vjp_backend": "ready_frontier"},
                                {"dependency_ready_shared_prefix_vjp": True,
                                 "shared_prefix_vjp_backend": "ready_frontier"}])
def test_scheduling_changes_no_gradient(kw):
    base = build_model(2)
    ref, early_ref, diag_ref = _run(copy.deepcopy(base))
    got, early, diag = _run(copy.deepcopy(base), **kw)
    for n in ref:
        torch.testing.assert_close(got[n], ref[n], rtol=1e-5, atol=1e-6, msg=n)
    assert early_ref == [0, 0, 0, 0] and diag_ref["autograd_calls"] == 3
    assert diag["finalized"] == 3
    if kw.get("dependency_ready_shared_prefix_vjp"):
        # the first subtree's node runs when its second group closes; the other child and the root
        # when the last group closes, all before the barrier
        assert early == [0, 1, 1, 3] and diag["finalized_before_barrier"] == 3
    else:
        assert early == [0, 0, 0, 0] and diag["finalized_before_barrier"] == 0
        # ready_frontier: the two children in one call, then the root
        assert diag["autograd_calls"] == 2


def test_unbuilt_shared_prefix_modes_are_refused():
    model = build_model(4)
    with pytest.raises(ConfigError):
        StreamingRun(model, boundary_cut=True, shared_prefix_vjp_backend="isolated_canonical")
    with pytest.raises(ConfigError):
        StreamingRun(model, boundary_cut=True, shared_prefix_vjp_mode="source_ready_serial")
