"""A caller-built ShardedOptimizerStep handed to the data-parallel trainer owns the step.

With ``sharded_step=`` the trainer materialises the group-count-scaled gradient into ``p.grad`` and lets
the ZeRO-1 step (reduction, clipping, shard-local optimizer, parameter broadcast) run it, as reference
src/thundersync/grpo/data_parallel.py:721-735 does. One process on the CPU: the result equals the
replicated torch-optimizer step, and gradient observers are refused on that path.
"""

from __future__ import annotations

import copy

import pytest
import torch

from tests.grpo_fixtures import build_model, make_batch
from thundersync_b200.engine.sharded_step import ShardedOptimizerStep
from thundersync_b200.engine.streaming import StreamingRun
from thundersync_b200.grpo.data_parallel import DataParallelThunderSync


def _factory(m):
    return StreamingRun(m, boundary_cut=True, stream_turns=False)


def _trainer(model, *, sharded: bool):
    named = [(n, p) for n, p in model.named_parameters() if p.requires_grad]
    kw = dict(run_factory=_factory, grad_clip=1.0, source_offload_mode="device_resident",
              source_offload_device=None)
    if sharded:
        shard = ShardedOptimizerStep(named, lambda ps: torch.optim.AdamW(ps, lr=1e-3, maximize=True),
                                     world_size=1, rank=0, grad_clip=1.0)
        return DataParallelThunderSync(model, shard.optimizer, sharded_step=shard, **kw)
    opt = torch.optim.AdamW([p for _, p in named], lr=1e-3, maximize=True)
    return DataParallelThunderSync(model, opt, **kw)


def _feed(dp, batch):
    for g, prompt, trajs in batch:
        dp.open_group(g, prompt)
        dp.register_group_trajectories(g, [t for t, _, _ in trajs])
        for tid, turns, reward in trajs:
            for tk, sc in turns:
                dp.append_turn(g, tid, tk, sc)
            dp.close_trajectory(tid, reward)
        dp.close_group(g)


def test_sharded_step_equals_the_replicated_step():
    base = build_model(51)
    batch, _ = make_batch(51, groups=2, per_group=3)
    out = []
    for sharded in (False, True):
        m = copy.deepcopy(base)
        dp = _trainer(m, sharded=sharded)
        _feed(dp, batch)
        stats = dp.step()
        assert ("sharded_step" in stats) is sharded and stats["global_grad_norm"] > 0
        out.append({n: p.detach().clone() for n, p in m.named_parameters()})
        assert all(p.grad is None for p in m.parameters() if p.requires_grad)
    for n in out[0]:
        torch.testing.assert_close(out[1][n], out[0][n], rtol=1e-6, atol=1e-7, msg=n)
    assert any(not torch.equal(out[0][n], p) for n, p in base.named_parameters())


def test_gradient_observers_are_refused_under_the_sharded_step():
    m = build_model(52)
    batch, _ = make_batch(52, groups=1, per_group=2)
    dp = _trainer(m, sharded=True)
    _feed(dp, batch)
    with pytest.raises(RuntimeError, match="observers"):
        dp.step(gradient_observer=lambda *a: None)


class _FailingBackward:
    def __init__(self, abort_error=None):
        self.aborted = False
        self.abort_error = abort_error

    def close_group(self, group_id):
        raise KeyError(group_id)

    def abort(self):
        self.aborted = True
        if self.abort_error is not None:
            raise self.abort_error


@pytest.mark.parametrize("abort_error", [None, OSError("abort failed")])
def test_a_failed_event_aborts_the_backward_and_reraises_its_own_error(abort_error):
    dp = _trainer(build_model(53), sharded=False)
    dp.bw = _FailingBackward(abort_error)
    before = dp._local_groups_closed
    with pytest.raises(KeyError) as raised:
        dp.close_group(3)
    assert dp.bw.aborted and dp._local_groups_closed == before
    notes = getattr(raised.value, "__notes__", [])
    assert (any("abort failed" in n for n in notes)) is (abort_error is not None)


def test_final_forest_configuration_rules():
    m = build_model(54)
    plain = DataParallelThunderSync(m, torch.optim.AdamW([p for p in m.parameters()], lr=1e-3),
                                    run_factory=_factory, source_offload_mode="device_resident",
                                    source_offload_device=None)
    with pytest.raises(ValueError, match="direct_when_group_bound"):
        plain.configure_final_forest(4096, 256)
    direct = DataParallelThunderSync(m, torch.optim.AdamW([p for p in m.parameters()], lr=1e-3),
                                     run_factory=_factory, source_offload_mode="device_resident",
                                     source_offload_device=None, direct_when_group_bound=True)
    assert not direct.final_forest_enabled
    with pytest.raises(RuntimeError, match="not configured"):
        direct.final_forest_max_tokens
    for cap, chunk in ((0, 256), (4096, 0)):
        with pytest.raises(ValueError, match="positive"):
            direct.configure_final_forest(cap, chunk)
    direct.configure_final_forest(4096, 256)
    assert direct.final_forest_enabled and direct.final_forest_max_tokens == 4096
