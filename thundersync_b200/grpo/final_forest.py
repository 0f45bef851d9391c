"""Final work as forest micro-batches (C33).

Once every reward of the step has landed each trajectory's advantage ``A_i``
is final, so the remaining objective ``Σ A_i S_i`` is linear and can run in
any grouping. Trajectories are packed group-whole under a token budget
(``pack_groups``); each micro-batch is compiled to a prefix-shared forest and
run once (``forest_logprobs``): a shared prompt is forwarded and backwarded
once per micro-batch. A micro-batch that runs out of memory is halved and
retried, and a single trajectory that still does not fit is rerun with
checkpointing and a bounded attention-output cache (reference:
src/thundersync/grpo/final_forest.py:182-434).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from thundersync_b200.engine.plan import compile_plan
from thundersync_b200.engine.segments import Segment, Trajectory, build_forest
from thundersync_b200.engine.step import forest_logprobs, split_by_trajectory
from thundersync_b200.grpo.packing import pack_groups
from thundersync_b200.ops.sink import GradSink, grad_sink

__all__ = ["FinalForestReport", "FinalItem", "backward_final_forest", "backward_claimed_payloads", "forest_trajectory",
           "forest_token_budget"]


@dataclass(frozen=True)
class FinalItem:
    group_id: int
    traj_id: int
    advantage: float
    prompt: tuple[int, ...]
    turns: tuple[tuple[tuple[int, ...], tuple[bool, ...]], ...]

    @property
    def n_tokens(self) -> int:
        return len(self.prompt) + sum(len(t) for t, _ in self.turns)


def forest_trajectory(item: FinalItem) -> Trajectory:
    segs = [Segment.prompt(item.prompt)]
    for tokens, scored in item.turns:
        # split a turn into maximal runs of equal scoring
        start = 0
        for i in range(1, len(tokens) + 1):
            if i == len(tokens) or scored[i] != scored[start]:
                run = tokens[start:i]
                segs.append(Segment.action(run) if scored[start] else Segment.observation(run))
                start = i
    return Trajectory(segs, group_id=item.group_id, traj_id=item.traj_id)


def forest_token_budget(device: torch.device, model: torch.nn.Module, *, fraction: float = 0.5) -> int:
    """Tokens per micro-batch that fit in ``fraction`` of free device memory."""
    if device.type != "cuda":
        return 1 << 16
    free, _ = torch.cuda.mem_get_info(device)
    cfg = model.config
    per_token = 2 * cfg.num_hidden_layers * (12 * cfg.hidden_size + 4 * cfg.intermediate_size)
    return max(1024, int(fraction * free / max(per_token, 1)))


def _microbatch(model, items: list[FinalItem], sink: GradSink | None, *, checkpoint: bool = False,
                cache=None, rows: int | None = None) -> None:
    trajs = [forest_trajectory(i) for i in items]
    plan = compile_plan(build_forest(trajs), device=next(model.parameters()).device)
    lp = forest_logprobs(model, plan, checkpoint=checkpoint, attention_cache=cache, rows=rows)
    per = split_by_trajectory(plan, lp)
    total = None
    for it in items:
        term = per[it.traj_id].sum() * it.advantage
        total = term if total is None else total + term
    if total is not None and total.requires_grad:
        with grad_sink(sink):
            total.backward()


@dataclass
class FinalForestReport:
    """What one final-forest call did (reference counterpart: src/thundersync/grpo/final_forest.py
    FinalForestReport)."""

    microbatches: int = 0
    halvings: int = 0
    checkpointed: int = 0
    out_of_memory: int = 0
    transactional: bool = False
    attention_cache: dict[str, int] | None = None


def _attention_cache_budget(device: torch.device) -> int:
    """A quarter of the memory the device could still hand out (free plus cached-but-unused)."""
    if device.type != "cuda":
        return 1 << 30
    free, _ = torch.cuda.mem_get_info(device)
    cached = torch.cuda.memory_reserved(device) - torch.cuda.memory_allocated(device)
    return (int(free) + max(0, int(cached))) // 4


def backward_final_forest(model, items: list[FinalItem], *, max_tokens_per_microbatch: int,
                          sink: GradSink | None = None, transactional: bool | None = None,
                          report: FinalForestReport | None = None, rows: int | None = None) -> int:
    """Backward ``Σ A_i S_i`` over ``items``; returns the number of micro-batches run.

    Memory ladder per micro-batch: run it as one forest; when that runs out of device memory, halve it
    (group-whole halves first) and retry; a single trajectory that still does not fit reruns with
    per-layer activation checkpointing, its attention outputs kept in a bounded cache so the backward's
    recompute skips the attention kernels (``AttentionOutputCache``, a quarter of the free memory).

    ``transactional`` (default: on whenever a sink is given): each micro-batch deposits into a private
    fp32 buffer that is added into the sink only once its backward completed, so a backward that runs out
    of memory part-way leaves the sink untouched and the retry neither loses nor double-counts any
    parameter's contribution (the reference resumes over the parameters the failed walk had not reached;
    this commits whole micro-batches instead).
    """
    from thundersync_b200.ops.attention import AttentionOutputCache
    from thundersync_b200.ops.fold import axpby_

    rep = report if report is not None else FinalForestReport()
    if transactional is None:
        transactional = sink is not None
    rep.transactional = bool(transactional and sink is not None)
    scratch = None
    if rep.transactional:
        scratch = torch.zeros_like(sink.buffer)
    batches = pack_groups(items, max_tokens_per_microbatch=max_tokens_per_microbatch, split_oversized_groups=True)
    queue = [(mb, False) for mb in batches]
    done = 0
    device = next(model.parameters()).device
    while queue:
        mb, ckpt = queue.pop(0)
        target = sink
        if scratch is not None:
            scratch.zero_()
            target = GradSink(sink.arena, scratch, scale=sink.scale)
        cache = AttentionOutputCache(_attention_cache_budget(device)) if ckpt else None
        try:
            _microbatch(model, mb, target, checkpoint=ckpt, cache=cache, rows=rows)
        except torch.OutOfMemoryError:
            rep.out_of_memory += 1
            if scratch is None and sink is not None:
                raise  # deposits may have landed in the shared sink: a retry could double-count them
            if device.type == "cuda":
                torch.cuda.empty_cache()
            if len(mb) > 1:
                half = len(mb) // 2
                queue[:0] = [(mb[:half], ckpt), (mb[half:], ckpt)]
                rep.halvings += 1
                continue
            if not ckpt:
                queue.insert(0, (mb, True))
                continue
            raise
        if scratch is not None:
            axpby_(sink.buffer, scratch, None, 1.0)
        done += 1
        rep.microbatches += 1
        if ckpt:
            rep.checkpointed += 1
            rep.attention_cache = cache.report()
    return done


def backward_claimed_payloads(trainer: Any, payloads: list[bytes]) -> None:
    """A thief runs claimed final trajectories into its own batch gradient."""
    from thundersync_b200.grpo.claims import decode_final_work

    items = []
    for p in payloads:
        gid, tid, adv, prompt, turns = decode_final_work(p)
        items.append(FinalItem(gid, tid, adv, tuple(prompt), tuple((tuple(t), tuple(s)) for t, s in turns)))
    cfg = getattr(trainer, "_final_forest", None)
    cap, rows = cfg if cfg else (1 << 16, None)
    sink = GradSink(trainer.arena, trainer.bw._main_grad())
    backward_final_forest(trainer.model, items, max_tokens_per_microbatch=cap, sink=sink, rows=rows)
