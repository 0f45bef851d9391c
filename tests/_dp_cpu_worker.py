"""torchrun worker for tests/test_dp_cpu.py (gloo, CPU fp32; not collected by pytest).

Modes:
  equality   each rank streams one group; DataParallelThunderSync.step() reduces a gradient equal to one
             process streaming both groups, divided by the group count
  unequal    rank 0 streams two groups, rank 1 one: the reduced gradient is the mean over all three
  broadcast  ranks build the model from different seeds; init_from_env leaves identical parameters
  guard      a step with an open group raises on every rank before any collective; after the group
             closes, the step runs and the replicas stay identical
Rank 0 writes a JSON verdict to --out.
"""

from __future__ import annotations

import argparse
import copy
import datetime
import json
import os
import sys
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

from tests.grpo_fixtures import EPS, build_model, make_batch  # noqa: E402
from thundersync_b200.engine.streaming import StreamingRun, arena_for  # noqa: E402
from thundersync_b200.grpo.data_parallel import DataParallelThunderSync  # noqa: E402
from thundersync_b200.grpo.reward_linear import RewardLinearBackward  # noqa: E402
from thundersync_b200.parallel.optimizer import FlatAdamW  # noqa: E402


def _factory(m):
    return StreamingRun(m, boundary_cut=True, stream_turns=False)


def _trainer(model):
    opt = FlatAdamW(arena_for(model), lr=1e-3, maximize=True)
    return DataParallelThunderSync.init_from_env(model, opt, run_factory=_factory, grad_clip=None,
                                                 source_offload_mode="device_resident", source_offload_device=None)


def _stream(dp, gid, prompt, trajs, close=True):
    dp.open_group(gid, prompt)
    dp.register_group_trajectories(gid, [t for t, _, _ in trajs])
    for tid, turns, reward in trajs:
        for tk, sc in turns:
            dp.append_turn(gid, tid, tk, sc)
        dp.close_trajectory(tid, reward)
    if close:
        dp.close_group(gid)


def _single(model, groups):
    run = StreamingRun(model, boundary_cut=True, stream_turns=False)
    bw = RewardLinearBackward(run, model, eps=EPS, source_offload_mode="device_resident", source_offload_device=None)
    for g, prompt, trajs in groups:
        bw.open_group(g, prompt, [t for t, _, _ in trajs])
        for tid, turns, reward in trajs:
            for tk, sc in turns:
                run.append_turn(g, tid, tk, sc)
            bw.close_trajectory(tid, reward)
        bw.close_group(g)
    bw.assert_safe_to_step(materialize=False)
    return bw.main_grad() / len(groups)


def _replicas_equal(model, world):
    h = torch.tensor([float(arena_for(model).flat.double().sum())], dtype=torch.float64)
    hs = [torch.zeros_like(h) for _ in range(world)]
    dist.all_gather(hs, h)
    return all(float(x) == float(hs[0]) for x in hs)


def mode_equality(rank, world, unequal=False):
    batch, _ = make_batch(0, groups=3 if unequal else world, per_group=4)
    model = build_model(1)
    ref = copy.deepcopy(model)
    dp = _trainer(model)
    mine = ([batch[0], batch[1]] if rank == 0 else [batch[2]]) if unequal else [batch[rank]]
    for g, prompt, trajs in mine:
        _stream(dp, g, prompt, trajs)
    captured = {}
    dp.step(gradient_observer=lambda tag, grad: captured.setdefault(tag, grad.clone()))
    got = captured["raw_reduced"]
    single = _single(ref, batch)
    rel = float((got[: single.numel()] - single).norm() / single.norm())
    return {"rel_err": rel, "replicas_equal": _replicas_equal(model, world)}


def mode_broadcast(rank, world):
    model = build_model(10 + rank)  # different on every rank before init
    _trainer(model)
    return {"replicas_equal": _replicas_equal(model, world)}


def mode_guard(rank, world):
    batch, _ = make_batch(0, groups=world, per_group=4)
    model = build_model(1)
    dp = _trainer(model)
    g, prompt, trajs = batch[rank]
    _stream(dp, g, prompt, trajs, close=False)
    raised = False
    try:
        dp.step()
    except RuntimeError:
        raised = True
    dp.close_group(g)
    dp.step()
    return {"raised": raised, "replicas_equal": _replicas_equal(model, world)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", required=True)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    rank, world = dist.get_rank(), dist.get_world_size()
    torch.manual_seed(0)
    res = {"equality": lambda: mode_equality(rank, world), "unequal": lambda: mode_equality(rank, world, True),
           "broadcast": lambda: mode_broadcast(rank, world), "guard": lambda: mode_guard(rank, world)}[args.mode]()
    flags = [None] * world
    dist.all_gather_object(flags, res)
    if rank == 0:
        Path(args.out).write_text(json.dumps({"ranks": flags, **res}))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
