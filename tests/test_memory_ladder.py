"""The close-rebuild memory ladder (plain -> blocked -> checkpoint -> checkpoint inputs on the host).

Reference behaviour: src/thundersync/engine/streaming.py:5160-5255 (rebuild rungs and their OOM retry)
and :2263-2316 (checkpoint-input host offload). Every rung must give the same gradient; an out-of-memory
error in a rebuild forward moves down one rung instead of failing the step (injected on the host here:
the rung's forward raises torch.cuda.OutOfMemoryError, so no device memory is ever exhausted).
"""

from __future__ import annotations

import pytest
import torch

from tests.grpo_fixtures import EPS, build_model, make_batch
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _grads(model, batch, order, run: StreamingRun):
    model.zero_grad(set_to_none=True)
    bw = RewardLinearBackward(run, model, eps=EPS)
    for g, prompt, trajs in batch:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
    for g, (tid, turns, reward) in order:
        for tk, sc in turns:
            run.append_turn(g, tid, tk, sc)
        bw.close_trajectory(tid, reward)
    for g, _, _ in batch:
        bw.close_group(g)
    bw.assert_safe_to_step()
    return {n: p.grad.detach().clone() for n, p in model.named_parameters()}


def _run(model, rung, **kw):
    run = StreamingRun(model, boundary_cut=True, stream_turns=False, rebuild_block_tokens=8, **kw)
    orig = run.rebuild_logprobs
    run.rebuild_logprobs = lambda ids, **k: orig(ids, **{**k, "executor": rung})
    return run


@pytest.mark.parametrize("rung", ["blocked", "checkpoint", "checkpoint_host"])
def test_every_rung_gives_the_plain_gradient(rung):
    model = build_model(11)
    batch, order = make_batch(11)
    ref_run = _run(model, "plain")
    ref = _grads(model, batch, order, ref_run)
    assert ref_run.rebuild_path_counts["plain"] > 0
    run = _run(model, rung)
    got = _grads(model, batch, order, run)
    for n in ref:
        torch.testing.assert_close(got[n], ref[n], rtol=1e-5, atol=5e-6, msg=n)
    counts = run.rebuild_path_counts
    assert counts[rung] > 0 or (rung == "blocked" and counts["plain"] > 0)


def test_out_of_memory_moves_one_rung_down():
    model = build_model(12)
    batch, order = make_batch(12)
    ref = _grads(model, batch, order, _run(model, "plain"))
    run = StreamingRun(model, boundary_cut=True, stream_turns=False, rebuild_block_tokens=8)
    real = run._rebuild_at
    failures = {"left": 2}

    def flaky(trajs, rung):
        if rung in ("plain", "blocked") and failures["left"] > 0:
            failures["left"] -= 1
            # a partial forward was built before the failure: the retry must not reuse it
            real(trajs, rung)
            raise torch.cuda.OutOfMemoryError("injected: the rung's activations do not fit")
        return real(trajs, rung)

    run._rebuild_at = flaky
    got = _grads(model, batch, order, run)
    for n in ref:
        torch.testing.assert_close(got[n], ref[n], rtol=1e-5, atol=5e-6, msg=n)
    counts = run.rebuild_path_counts
    assert counts["oom_retries"] == 2 and counts["checkpoint"] >= 2


def test_explicit_rung_does_not_retry():
    model = build_model(13)
    batch, order = make_batch(13)
    run = _run(model, "checkpoint")

    def oom(trajs, rung):
        raise torch.cuda.OutOfMemoryError("injected")

    run._rebuild_at = oom
    with pytest.raises(torch.cuda.OutOfMemoryError):
        _grads(model, batch, order, run)


def test_memory_report_shape_without_a_device():
    model = build_model(14)
    run = StreamingRun(model, boundary_cut=True, stream_turns=False)
    rep = run.turn_memory_report
    assert rep["windows"] == {} and rep["oom_retries"] == 0
    assert run.turn_memory_windows == []
    diag = run.rebuild_checkpoint_offload_diagnostics()
    assert diag["write_bytes"] == 0 and diag["read_bytes"] == 0
    shape = run._turn_memory_shape()
    assert shape["plain_activation"] > shape["checkpoint_activation"] > shape["host_checkpoint_activation"] > 0


def test_several_branches_rebuild_apart_unless_backwarded_jointly():
    """Without joint_backward each branch's graph is its own: per-branch backwards all work; with it the
    branches share one pack and one backward. Both give the same log-probs."""
    import copy

    from tests.grpo_fixtures import build_model, make_batch
    from thundersync_b200.engine.streaming import StreamingRun

    base = build_model(61)
    batch, _ = make_batch(61, groups=1, per_group=3)
    g, prompt, trajs = batch[0]
    out = []
    for joint in (False, True):
        m = copy.deepcopy(base)
        run = StreamingRun(m, boundary_cut=True, stream_turns=False)
        run.open_group(g, prompt)
        for tid, turns, _ in trajs:
            for tk, sc in turns:
                run.append_turn(g, tid, tk, sc)
        tids = [t for t, _, _ in trajs]
        lps = run.rebuild_logprobs(tids, joint_backward=joint, releasing_bytes=lambda: 1 << 20)
        if joint:
            sum(lp.sum() for lp in lps).backward()
        else:
            for lp in lps:
                lp.sum().backward()  # one branch at a time
        out.append(([lp.detach() for lp in lps], {n: p.grad.clone() for n, p in m.named_parameters()
                                                   if p.grad is not None}))
    for a, b in zip(out[0][0], out[1][0]):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
    for n in out[0][1]:
        torch.testing.assert_close(out[0][1][n], out[1][1][n], rtol=1e-5, atol=1e-6)
