"""Forest step: physical-forest forward and gathered log-probs (C08, C09).

``forest_logprobs(model, plan)`` runs the native executor once over the plan's
physical token stream; each node is a segment whose attention reads its
ancestors' spans of the same pass (``Segment.key_ranges``), causal only within
itself. Only the predecessors of scored tokens reach the fused LM head, and
the result is indexed logically (``logical_to_slot``) so shared positions
receive the sum of their logical uses' gradients from autograd. Mirrors
reference src/thundersync/engine/step.py:383-470.
"""

from __future__ import annotations

import contextlib
from dataclasses import dataclass
from typing import Any

import torch

from thundersync_b200.engine.layers import Segment, executor_for, spec_of
from thundersync_b200.engine.plan import ExecutionPlan
from thundersync_b200.engine.streaming import arena_for
from thundersync_b200.ops.logprob import lm_head_logprob

__all__ = ["forest_logprobs", "split_by_trajectory", "assert_supported", "base_model", "unembedding",
           "hybrid_layer_kinds", "StepStats", "forest_context", "bound_plan"]


@dataclass
class StepStats:
    physical_tokens: int
    logical_tokens: int
    scored_rows: int
    logical_scored: int


def base_model(model: torch.nn.Module) -> torch.nn.Module:
    inner = getattr(model, "model", None)
    if inner is None or not hasattr(inner, "layers"):
        raise TypeError("expected a causal LM with .model.layers")
    return inner


def unembedding(model: torch.nn.Module) -> torch.Tensor:
    head = getattr(model, "lm_head", None)
    if head is None:
        raise TypeError("expected a causal LM with .lm_head")
    return getattr(head, "base_layer", head).weight


def hybrid_layer_kinds(model: torch.nn.Module) -> list[str]:
    return list(spec_of(model).kinds)


def assert_supported(model: torch.nn.Module, *, allow_hybrid: bool = False) -> None:
    """Refuse models the executor cannot run (recurrent layers off the streaming path)."""
    base_model(model)
    unembedding(model)
    kinds = set(spec_of(model).kinds)
    unknown = kinds - {"full_attention", "linear_attention"}
    if unknown:
        raise NotImplementedError(f"unsupported layer kinds {sorted(unknown)}")
    if "linear_attention" in kinds and not allow_hybrid:
        raise NotImplementedError(
            "recurrent (linear-attention) layers carry state along one chain; the forest path "
            "shares nodes across branches and is not defined for them -- use StreamingRun"
        )


def _run_checkpointed(ex, ids: torch.Tensor, pos: torch.Tensor, segs: list[Segment], cache) -> torch.Tensor:
    """Per-layer activation checkpointing over one forest pass; attention outputs may come from ``cache``."""
    from torch.utils.checkpoint import checkpoint

    h = ex.embed(ids)
    for i, kind in enumerate(ex.spec.kinds):
        fn = ex.attention_layer if kind == "full_attention" else ex.linear_layer

        def body(h_in, _i=i, _fn=fn):
            ctx = cache.layer(_i) if cache is not None else contextlib.nullcontext()
            with ctx:
                return _fn(_i, h_in, pos, segs)[0]

        h = checkpoint(body, h, use_reentrant=False)
    return ex.final_norm(h)


def forest_logprobs(model: torch.nn.Module, plan: ExecutionPlan | None = None, *, gate: bool = True,
                    stats: list[StepStats] | None = None, checkpoint: bool = False,
                    attention_cache: Any = None, rows: int | None = None) -> torch.Tensor:
    """Log-probs of the plan's scored tokens. ``checkpoint`` keeps only layer inputs for the backward
    (each layer is recomputed there); an :class:`~thundersync_b200.ops.attention.AttentionOutputCache`
    lets that recompute reuse attention outputs within its byte budget. ``plan=None`` runs the plan that
    :func:`forest_context` bound for the model's device; ``rows`` sets the LM head's rows per block."""
    assert_supported(model)
    dev = next(model.parameters()).device
    if plan is None:
        plan = bound_plan(dev)
        if plan is None:
            raise RuntimeError("forest_logprobs without a plan needs one bound by forest_context")
    plan = plan.to(dev)
    ex = executor_for(model, arena_for(model))
    segs = []
    for n in range(plan.n_nodes):
        s, e = int(plan.node_start[n]), int(plan.node_end[n])
        if e > s:
            segs.append((s, Segment(s, e - s, [], plan.key_ranges[n][:-1])))
    segs = [sg for _, sg in sorted(segs, key=lambda x: x[0])]
    if checkpoint and torch.is_grad_enabled():
        h = _run_checkpointed(ex, plan.token_ids, plan.position_ids, segs, attention_cache)
    else:
        h, _ = ex.run(plan.token_ids, plan.position_ids, segs)
    w = ex.head_weight()
    if gate:
        kw = {} if rows is None else {"rows": rows}
        lp = lm_head_logprob(h.index_select(0, plan.score_src), w, plan.score_tgt, **kw)
    else:  # measurement mode: project every position, then gather
        lp_all = torch.log_softmax(h.float() @ w.float().t(), -1)
        lp = lp_all[plan.score_src].gather(-1, plan.score_tgt[:, None]).squeeze(-1)
    if stats is not None:
        stats.append(StepStats(plan.n_physical, plan.forest.logical_tokens, plan.n_scored, plan.n_logical_scored))
    return lp.index_select(0, plan.logical_to_slot)


def split_by_trajectory(plan: ExecutionPlan, logical: torch.Tensor) -> dict[int, torch.Tensor]:
    out: dict[int, torch.Tensor] = {}
    traj = plan.logical_traj.tolist()
    start = 0
    for i in range(1, len(traj) + 1):
        if i == len(traj) or traj[i] != traj[start]:
            out[traj[start]] = logical[start:i]
            start = i
    for t in plan.forest.trajectories:
        out.setdefault(t.traj_id, logical.new_zeros(0))
    return out


_BOUND: dict[str, ExecutionPlan] = {}


def _device_key(device: torch.device | str) -> str:
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    return str(d)


def bound_plan(device: torch.device | str) -> ExecutionPlan | None:
    """The plan :func:`forest_context` bound for ``device`` (None outside one)."""
    return _BOUND.get(_device_key(device))


@contextlib.contextmanager
def forest_context(plan: ExecutionPlan):
    """Bind ``plan`` to its device for a forward, or a whole step (forward, loss, backward), so that
    :func:`forest_logprobs` called without a plan runs it. Contexts nest: leaving one restores the plan
    bound before it. The executor itself takes the plan as an argument, so a checkpointed recompute in
    the backward needs no binding (reference src/thundersync/engine/step.py:142-164 binds the plan for
    its attention-interface dispatch instead)."""
    key = _device_key(plan.token_ids.device)
    previous = _BOUND.get(key)
    _BOUND[key] = plan
    try:
        yield plan
    finally:
        if previous is None:
            _BOUND.pop(key, None)
        else:
            _BOUND[key] = previous


def register_attention() -> None:
    """API parity: the forest path calls the native executor directly."""
    return None
