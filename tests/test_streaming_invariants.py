"""Streaming invariants on CPU fp32 (the reference's streaming-exactness battery, restated for this engine).

Each test runs the same GRPO batch through the streaming engine twice under two settings that must
not change the gradient: trajectory arrival order, per-layer activation checkpointing, source offload
placement, rebuild block size, chunked key/value streaming, parameter-adjoint reduction order.
"""

from __future__ import annotations

import copy

import pytest
import torch

from tests.grpo_fixtures import EPS, build_model, make_batch
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.reward_linear import RewardLinearBackward


def _grads(model, batch, order, *, run_kw=None, bw_kw=None, binary=False, stream_turns=False):
    model.zero_grad(set_to_none=True)
    run = StreamingRun(model, boundary_cut=True, stream_turns=stream_turns, **(run_kw or {}))
    bw = RewardLinearBackward(run, model, eps=EPS, **(bw_kw or {}))
    if binary:
        bw.configure_binary_rewards()
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


def _close(a, b, rtol=1e-5, atol=5e-6):
    assert a.keys() == b.keys()
    for n in a:
        torch.testing.assert_close(a[n], b[n], rtol=rtol, atol=atol, msg=n)


def _orders(order):
    """The fixture's shuffled order, its reverse, and a round-robin interleave across groups."""
    by_group: dict[int, list] = {}
    for g, item in order:
        by_group.setdefault(g, []).append((g, item))
    rr = []
    while any(by_group.values()):
        for g in sorted(by_group):
            if by_group[g]:
                rr.append(by_group[g].pop(0))
    return [order, list(reversed(order)), rr]


@pytest.mark.parametrize("binary", [False, True])
def test_gradient_independent_of_arrival_order(binary):
    model = build_model(3)
    batch, order = make_batch(3)
    res = [_grads(copy.deepcopy(model), batch, o, binary=binary) for o in _orders(order)]
    _close(res[0], res[1])
    _close(res[0], res[2])


def test_checkpointed_executor_matches_plain():
    model = build_model(4)
    batch, order = make_batch(4)
    a = _grads(copy.deepcopy(model), batch, order)
    b = _grads(copy.deepcopy(model), batch, order, run_kw={"checkpoint": True})
    _close(a, b, rtol=0, atol=0)  # recomputation on CPU repeats the same arithmetic: bitwise


def test_source_offload_modes_agree():
    model = build_model(5)
    batch, order = make_batch(5)
    a = _grads(copy.deepcopy(model), batch, order, bw_kw={"source_offload_mode": "blocking"})
    b = _grads(copy.deepcopy(model), batch, order, bw_kw={"source_offload_mode": "device_resident",
                                                          "source_offload_device": None})
    _close(a, b)


@pytest.mark.parametrize("block", [8, 64])
def test_rebuild_block_size_does_not_change_gradient(block):
    model = build_model(6)
    batch, order = make_batch(6, multi_turn=True)
    a = _grads(copy.deepcopy(model), batch, order, stream_turns=True)
    b = _grads(copy.deepcopy(model), batch, order, stream_turns=True, run_kw={"rebuild_block_tokens": block})
    _close(a, b)


def test_turn_streaming_matches_whole_trajectories():
    model = build_model(7)
    batch, order = make_batch(7, multi_turn=True)
    a = _grads(copy.deepcopy(model), batch, order, stream_turns=True)
    b = _grads(copy.deepcopy(model), batch, order, stream_turns=False)
    _close(a, b, rtol=2e-4, atol=2e-6)


@pytest.mark.parametrize("reduction", ["arrival", "canonical_source"])
def test_parameter_adjoint_reduction_modes(reduction):
    model = build_model(8)
    batch, order = make_batch(8)
    a = _grads(copy.deepcopy(model), batch, order)
    b = _grads(copy.deepcopy(model), batch, order, run_kw={"parameter_adjoint_reduction": reduction})
    _close(a, b)


@pytest.mark.parametrize("kw,msg", [
    ({"turn_boundary_rebuild": True, "stream_turns": False}, "stream_turns"),
    ({"chunk": 0}, "chunk"),
    ({"rebuild_block_tokens": 0}, "rebuild_block_tokens"),
    ({"boundary_adjoint_backend": "cuda_graph"}, "boundary_adjoint_backend"),
    ({"boundary_adjoint_max_degree": 17}, "boundary_adjoint_max_degree"),
    ({"shared_prefix_vjp_mode": "eager"}, "shared_prefix_vjp_mode"),
    ({"parameter_adjoint_reduction": "sorted"}, "parameter_adjoint_reduction"),
])
def test_streaming_run_refuses_bad_settings(kw, msg):
    model = build_model(0)
    kw = dict(kw)
    stream_turns = kw.pop("stream_turns", True)
    with pytest.raises((ValueError, NotImplementedError), match=msg.split("_")[0]):
        StreamingRun(model, boundary_cut=True, stream_turns=stream_turns, **kw)


def test_shared_prefix_timing_and_adjoint_storage_diagnostics():
    model = build_model(9)
    batch, order = make_batch(9)
    a = _grads(copy.deepcopy(model), batch, order, run_kw={"parameter_adjoint_reduction": "canonical_source"})
    m = copy.deepcopy(model)
    b = _grads(m, batch, order, run_kw={"parameter_adjoint_reduction": "canonical_source",
                                        "parameter_adjoint_storage_device": "cpu",
                                        "shared_prefix_vjp_timing": True})
    _close(a, b, rtol=0, atol=0)


def test_rebuild_reserve_option_is_accepted_on_cpu():
    model = build_model(10)
    batch, order = make_batch(10, multi_turn=True)
    a = _grads(copy.deepcopy(model), batch, order, stream_turns=True)
    b = _grads(copy.deepcopy(model), batch, order, stream_turns=True,
               run_kw={"rebuild_plain_reserve_bytes": 1 << 30, "rebuild_block_tokens": 8})
    _close(a, b)


@pytest.mark.parametrize("binary", [False, True])
def test_combined_known_reward_sources_give_the_same_gradient(binary):
    """Closes of one group that share a reward run as one packed source; the gradient is unchanged."""
    model = build_model(21)
    batch, _ = make_batch(21)

    def grads(combine):
        model.zero_grad(set_to_none=True)
        run = StreamingRun(model, boundary_cut=True, stream_turns=False)
        bw = RewardLinearBackward(run, model, eps=EPS, combine_known_reward_sources=combine)
        if binary:
            bw.configure_binary_rewards()
        for g, prompt, trajs in batch:
            bw.open_group(g, prompt, [t for t, _, _ in trajs])
        for g, _, trajs in batch:
            items = []
            for j, (tid, turns, reward) in enumerate(trajs):
                for tk, sc in turns:
                    run.append_turn(g, tid, tk, sc)
                r = float(j % 2) if binary else (0.25 if j % 2 else 0.75)
                items.append((tid, r))
            bw.close_trajectories(items)
            bw.close_group(g)
        bw.assert_safe_to_step()
        return {n: p.grad.detach().clone() for n, p in model.named_parameters()}, bw.source_offload_report

    ref, r0 = grads(False)
    got, r1 = grads(True)
    assert r0["combined_sources"] == 0 and r1["combined_sources"] > 0 and r1["sources"] < r0["sources"]
    _close(got, ref)


def test_concatenating_baseline_keeps_chains_and_same_logprobs():
    """``chunked_sdpa=False`` (the memory gate's baseline) keeps each pack's concatenated K/V chains alive with
    its graph, and changes no number: log-probs and gradients equal the streamed path's."""
    import copy

    from tests.grpo_fixtures import build_model
    from thundersync_b200.engine.streaming import StreamingRun

    base = build_model(11)
    out = []
    for chunked in (True, False):
        model = copy.deepcopy(base)
        run = StreamingRun(model, chunked_sdpa=chunked)
        run.open_group(0, [1, 2, 3, 4, 5])
        run.append_turn(0, 0, [6, 7, 8], [True, True, True])
        run.append_turn(0, 0, [9, 10], [True, False])
        lp = run.logprobs(0)
        if not chunked:
            kept = [t for t in run._trajs[0].logprobs if t.grad_fn is not None]
            assert kept, "turn log-probs carry a graph"
        lp.sum().backward()
        out.append((lp.detach().clone(), {n: p.grad.clone() for n, p in model.named_parameters()}))
        run.close()
    torch.testing.assert_close(out[0][0], out[1][0])
    for n in out[0][1]:
        torch.testing.assert_close(out[0][1][n], out[1][1][n])


def test_lm_head_row_block_changes_blocks_not_results(monkeypatch):
    """``StreamingRun(chunk=...)`` sets the LM head's rows per block; the values and gradients stay."""
    import thundersync_b200.engine.streaming as S
    from thundersync_b200.ops.logprob import _row_block

    assert _row_block(1, True) == 128 and _row_block(129, True) == 256 and _row_block(3, False) == 3
    with pytest.raises(ValueError):
        _row_block(0, False)
    seen = []
    real = S.lm_head_logprob

    def spy(h, w, t, *, rows):
        seen.append(rows)
        return real(h, w, t, rows=rows)

    monkeypatch.setattr(S, "lm_head_logprob", spy)
    model = build_model(41)
    batch, order = make_batch(41, groups=1, per_group=3)
    res = []
    for chunk in (None, 3):
        m = copy.deepcopy(model)
        res.append(_grads(m, batch, order, run_kw={"chunk": chunk}, stream_turns=True))
    assert 2048 in seen and 3 in seen
    _close(res[0], res[1])
    with pytest.raises(ValueError):
        StreamingRun(model, chunk=0)


@pytest.mark.parametrize("backend,degree", [("native", 1), ("native", 2), ("triton", 16)])
def test_boundary_adjoint_backend_stages_contributions_without_changing_the_gradient(backend, degree):
    """Staged ledgers (reduced in arrival order when max_degree wait or the ledger is read) equal the
    immediate fp32 adds bitwise (CPU: the same sequential adds)."""
    model = build_model(42)
    batch, order = make_batch(42, groups=2, per_group=4, multi_turn=True)
    ref = _grads(copy.deepcopy(model), batch, order, stream_turns=True)
    got = _grads(copy.deepcopy(model), batch, order, stream_turns=True,
                 run_kw={"boundary_adjoint_backend": backend, "boundary_adjoint_max_degree": degree})
    for n in ref:
        assert torch.equal(ref[n], got[n]), n


def test_boundary_ledger_flushes_at_max_degree_and_on_read():
    from thundersync_b200.engine.boundary import Boundary

    real = [torch.randn(3, 4, requires_grad=True)]
    b = Boundary.cut([r * 1.0 for r in real], reduce_backend="native", max_degree=3)
    parts = [torch.randn(3, 4, dtype=torch.bfloat16) for _ in range(5)]
    for x in parts[:2]:
        b.accumulate_explicit([x])
    assert b.has_adjoint() and b._ledgers[0] is None and len(b._pending[0]) == 2
    b.accumulate_explicit([parts[2]])  # the third waiting contribution triggers the reduction
    assert b._pending[0] == [] and b._ledgers[0].dtype == torch.float32
    for x in parts[3:]:
        b.accumulate_explicit([x])
    (led,) = b.peek()
    want = torch.zeros(3, 4)
    for x in parts:
        want += x.float()
    assert torch.equal(led, want)
    with pytest.raises(ValueError):
        Boundary.cut([torch.randn(2, requires_grad=True) * 1.0], reduce_backend="native", max_degree=17)
