"""Final work as forest micro-batches (C33).

Once every reward of the step has landed each trajectory's advantage ``A_i``
is final, so the remaining objective ``Σ A_i S_i`` is linear and can run in
any grouping. Trajectories are packed group-whole under a token budget
(``pack_groups``); each micro-batch is compiled to a prefix-shared forest and
run once (``forest_logprobs``): a shared prompt is forwarded and backwarded
once per micro-batch. A micro-batch that runs out of memory is halved and
retried (reference: src/thundersync/grpo/final_forest.py:246-434).
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

__all__ = ["FinalItem", "backward_final_forest", "backward_claimed_payloads", "forest_trajectory", "forest_token_budget"]


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


def _microbatch(model, items: list[FinalItem], sink: GradSink | None) -> None:
    trajs = [forest_trajectory(i) for i in items]
    plan = compile_plan(build_forest(trajs), device=next(model.parameters()).device)
    lp = forest_logprobs(model, plan)
    per = split_by_trajectory(plan, lp)
    total = None
    for it in items:
        term = per[it.traj_id].sum() * it.advantage
        total = term if total is None else total + term
    if total is not None and total.requires_grad:
        with grad_sink(sink):
            total.backward()


def backward_final_forest(model, items: list[FinalItem], *, max_tokens_per_microbatch: int,
                          sink: GradSink | None = None) -> int:
    """Backward ``Σ A_i S_i`` over ``items``; returns the number of micro-batches run."""
    batches = pack_groups(items, max_tokens_per_microbatch=max_tokens_per_microbatch, split_oversized_groups=True)
    done = 0
    queue = list(batches)
    while queue:
        mb = queue.pop(0)
        try:
            _microbatch(model, mb, sink)
            done += 1
        except torch.OutOfMemoryError:
            if len(mb) == 1:
                raise
            half = len(mb) // 2
            queue[:0] = [mb[:half], mb[half:]]
            torch.cuda.empty_cache()
    return done


def backward_claimed_payloads(trainer: Any, payloads: list[bytes]) -> None:
    """A thief runs claimed final trajectories into its own batch gradient."""
    from thundersync_b200.grpo.claims import decode_final_work

    items = []
    for p in payloads:
        gid, tid, adv, prompt, turns = decode_final_work(p)
        items.append(FinalItem(gid, tid, adv, tuple(prompt), tuple((tuple(t), tuple(s)) for t, s in turns)))
    cap = trainer._final_forest[0] if getattr(trainer, "_final_forest", None) else 1 << 16
    sink = GradSink(trainer.arena, trainer.bw._main_grad())
    backward_final_forest(trainer.model, items, max_tokens_per_microbatch=cap, sink=sink)
