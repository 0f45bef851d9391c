"""torchrun worker for tests/test_dp_gpu.py (not collected by pytest).

Modes:
  equality   2 ranks x 1 group each through DataParallelThunderSync.step() equal
             one process streaming both groups (fp32 tiny model on CUDA,
             gradients averaged over groups), native reduction path.
  native     the symmetric-memory all-reduce is bitwise equal on every rank and
             equals a fixed-order host sum; reduce-scatter + fused AdamW gather
             leaves identical parameters on every rank.
  timeout    a barrier whose peer never arrives sets the status word (bounded).
  sharded    the ZeRO-1 step (FlatAdamW.sharded: native reduce-scatter, fused AdamW on each shard,
             bf16 parameter gather into every rank) leaves every rank with the parameters one
             replicated FlatAdamW step produces from the same averaged gradient.
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

from tests.grpo_fixtures import EPS, make_batch  # noqa: E402
from thundersync_b200.engine.streaming import StreamingRun, arena_for  # noqa: E402
from thundersync_b200.grpo.data_parallel import DataParallelThunderSync  # noqa: E402
from thundersync_b200.grpo.reward_linear import RewardLinearBackward  # noqa: E402
from thundersync_b200.models.qwen3 import PRESETS, Qwen3ForCausalLM  # noqa: E402
from thundersync_b200.parallel.optimizer import FlatAdamW  # noqa: E402

CFG = PRESETS["qwen3-1.7b"].with_(num_hidden_layers=2, hidden_size=256, intermediate_size=512,
                                  num_attention_heads=4, num_key_value_heads=2, vocab_size=1024)


def _model(seed, device, dtype):
    torch.manual_seed(seed)
    with torch.device(device):
        m = Qwen3ForCausalLM(CFG)
    return m.to(dtype=dtype)


def _stream(trainer, gid, prompt, trajs, order):
    trainer.open_group(gid, prompt)
    trainer.register_group_trajectories(gid, [t for t, _, _ in trajs])
    for tid, turns, reward in [x for x in order]:
        for tk, sc in turns:
            trainer.append_turn(gid, tid, tk, sc)
        trainer.close_trajectory(tid, reward)
    trainer.close_group(gid)


def mode_equality(rank, world, device):
    batch, _ = make_batch(0, groups=world, per_group=4, vocab=CFG.vocab_size, lo=40, hi=120, prompt_len=64)
    model = _model(1, device, torch.bfloat16)
    ref = copy.deepcopy(model)
    opt = FlatAdamW(arena_for(model), lr=1e-3, maximize=True)
    run_factory = lambda m: StreamingRun(m, boundary_cut=True, stream_turns=False)  # noqa: E731
    dp = DataParallelThunderSync.init_from_env(model, opt, run_factory=run_factory, grad_clip=None,
                                               source_offload_mode="device_resident", source_offload_device=None)
    g, prompt, trajs = batch[rank]
    _stream(dp, g, prompt, trajs, trajs)
    captured = {}
    stats = dp.step(gradient_observer=lambda tag, grad: captured.setdefault(tag, grad.clone()))
    dp_grad = captured["raw_reduced"]
    # single process over both groups
    run = StreamingRun(ref, boundary_cut=True, stream_turns=False)
    bw = RewardLinearBackward(run, ref, eps=EPS, source_offload_mode="device_resident", source_offload_device=None)
    for g2, prompt2, trajs2 in batch:
        bw.open_group(g2, prompt2, [t for t, _, _ in trajs2])
        for tid, turns, reward in trajs2:
            for tk, sc in turns:
                run.append_turn(g2, tid, tk, sc)
            bw.close_trajectory(tid, reward)
        bw.close_group(g2)
    bw.assert_safe_to_step(materialize=False)
    single = bw.main_grad() / len(batch)
    rel = float((dp_grad[: single.numel()] - single).norm() / single.norm())
    # replicas identical after the step
    h = torch.tensor([float(arena_for(model).flat.float().sum())], device=device, dtype=torch.float64)
    hs = [torch.zeros_like(h) for _ in range(world)]
    dist.all_gather(hs, h)
    return {"rel_err": rel, "path": stats.get("reduction_path"), "replicas_equal": all(float(x) == float(hs[0]) for x in hs),
            "norm": stats["global_grad_norm"]}


def mode_sharded(rank, world, device):
    batch, _ = make_batch(0, groups=world, per_group=4, vocab=CFG.vocab_size, lo=40, hi=120, prompt_len=64)
    model = _model(1, device, torch.bfloat16)
    ref = copy.deepcopy(model)
    opt = FlatAdamW.sharded(arena_for(model), lr=1e-3, maximize=True)
    run_factory = lambda m: StreamingRun(m, boundary_cut=True, stream_turns=False)  # noqa: E731
    dp = DataParallelThunderSync.init_from_env(model, opt, run_factory=run_factory, grad_clip=1.0,
                                               source_offload_mode="device_resident", source_offload_device=None)
    g, prompt, trajs = batch[rank]
    _stream(dp, g, prompt, trajs, trajs)
    captured = {}
    stats = dp.step(gradient_observer=lambda tag, grad: captured.setdefault(tag, grad.clone()))
    torch.cuda.synchronize()
    # the reduce-scatter leaves only this rank's shard reduced: gather the shards into the full mean gradient
    arena = arena_for(model)
    lo, hi = opt.lo, opt.hi
    full = torch.zeros(arena.numel, device=device, dtype=torch.float32)
    full[lo:hi] = captured["raw_reduced"][lo:hi]
    dist.all_reduce(full)
    # one replicated update from the same gradient
    ref_arena = arena_for(ref)
    ref_opt = FlatAdamW(ref_arena, lr=1e-3, maximize=True)
    from thundersync_b200.parallel.optimizer import global_sq_norm

    coef, nrm = ref_opt.clip_coefficient(global_sq_norm(full), 1.0)
    ref_opt.step(full, clip_coef=coef)
    torch.cuda.synchronize()
    diff = float((arena.flat.float() - ref_arena.flat.float()).abs().max())
    h = torch.tensor([float(arena.flat.float().sum())], device=device, dtype=torch.float64)
    hs = [torch.zeros_like(h) for _ in range(world)]
    dist.all_gather(hs, h)
    return {"max_param_diff": diff, "path": stats.get("reduction_path"), "norm": stats["global_grad_norm"],
            "ref_norm": float(nrm), "replicas_equal": all(float(x) == float(hs[0]) for x in hs)}


def mode_native(rank, world, device):
    from thundersync_b200.parallel.symm import SymmetricWorkspace, shard_bounds

    ws = SymmetricWorkspace(device)
    n = 1_000_003
    buf, ptrs = ws.alloc(n + 64, torch.float32)
    gen = torch.Generator().manual_seed(100 + rank)
    mine = torch.randn(n, generator=gen)
    buf[:n].copy_(mine.to(device))
    buf[n:].zero_()
    ws.all_reduce_mean(buf, ptrs, pre_scale=0.5)
    torch.cuda.synchronize()
    ws.check()
    # host fixed-order reference
    parts = [torch.randn(n, generator=torch.Generator().manual_seed(100 + r)) for r in range(world)]
    acc = parts[0].clone()
    for p in parts[1:]:
        acc += p
    ref = acc * (0.5 / world)
    got = buf[:n].cpu()
    close = bool(torch.allclose(got, ref, rtol=1e-6, atol=1e-6))
    d = torch.tensor([float(got.double().sum())], device=device, dtype=torch.float64)
    ds = [torch.zeros_like(d) for _ in range(world)]
    dist.all_gather(ds, d)
    bitwise_same = all(float(x) == float(ds[0]) for x in ds)
    # one-shot all-reduce: same fixed rank order, so bitwise equal to the two-shot result
    small = 70_001
    sbuf, sptrs = ws.alloc(small, torch.float32)
    sbuf.copy_(mine[:small].to(device))
    out = torch.empty(small, device=device)
    ws.all_reduce_mean_oneshot(sbuf, sptrs, out, pre_scale=0.5)
    torch.cuda.synchronize()
    ws.check()
    ws.all_reduce_mean(sbuf, sptrs, pre_scale=0.5)  # the two-shot over the same (unchanged) input
    torch.cuda.synchronize()
    ws.check()
    oneshot_equal = bool(torch.equal(out, sbuf)) and bool(torch.allclose(out.cpu(), ref[:small], rtol=1e-6, atol=1e-6))
    # reduce-scatter + fused AdamW gather
    model = _model(2, device, torch.bfloat16)
    arena = arena_for(model)
    flat, pptrs = ws.alloc(arena.numel, arena.dtype)
    arena.rehome(flat)
    opt = FlatAdamW(arena, lr=1e-2, shard=shard_bounds(arena.numel, world, rank), maximize=True)
    gbuf, gptrs = ws.alloc(-(-arena.numel // (4 * world)) * 4 * world, torch.float32)
    gbuf.copy_(torch.randn(gbuf.numel(), generator=torch.Generator().manual_seed(7 + rank)).to(device))
    ws.reduce_scatter(gbuf, gptrs)
    opt.step_gather(gbuf[opt.lo:opt.hi], pptrs, ws.norm_slots, 1.0)
    ws.barrier(2)
    torch.cuda.synchronize()
    ws.check()
    s = torch.tensor([float(arena.flat.float().double().sum())], device=device, dtype=torch.float64)
    ss = [torch.zeros_like(s) for _ in range(world)]
    dist.all_gather(ss, s)
    return {"allreduce_close": close, "allreduce_bitwise_same": bitwise_same, "oneshot_equal": oneshot_equal,
            "params_same_after_gather": all(float(x) == float(ss[0]) for x in ss)}


def mode_timeout(rank, world, device):
    from thundersync_b200.parallel.symm import SymmetricWorkspace

    ws = SymmetricWorkspace(device, timeout_s=0.2)
    dist.barrier()
    code = 0
    if rank == 0:
        # rank 0 enters a barrier slot that rank 1 never enters: bounded wait, status set
        ws.barrier(5)
        torch.cuda.synchronize()
        code = int(ws.status.item())
    dist.barrier()
    return {"status_code": code}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--mode", required=True)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        res = {"equality": mode_equality, "native": mode_native, "timeout": mode_timeout,
               "sharded": mode_sharded}[a.mode](rank, world, device)
        if rank == 0:
            Path(a.out).write_text(json.dumps(res))
    finally:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
