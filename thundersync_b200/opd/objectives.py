"""On-policy distillation objectives (C36).

Both objectives minimise the sampled reverse KL of the student against a
frozen teacher, per scored token ``t``:

    loss_t = w_t * exp(lp_t - sg(lb_t)) * sg(lb_t - lq_t)

with ``lp`` the student's log-prob (graph-attached), ``lb`` its behaviour
(old) log-prob -- bitwise the same value at epoch 1, so the ratio is 1 and
the gradient is ``w_t (lb_t - lq_t) grad lp_t`` -- and ``lq`` the teacher's.
The batch gradient is divided by the scored-token mass (``token_mean``) at
``assert_safe_to_step``. The teacher coefficient is a constant, so every
backward goes straight into ``param.grad``; the prompt is backwarded once
per group through the run's boundary cut.

* :class:`OPDTurnStream` backwards each turn as soon as its teacher scores
  arrive (``StreamingRun(turn_boundary_rebuild=True)`` cuts each turn's
  outgoing state) and replays the deferred state adjoints in reverse at
  trajectory close.
* :class:`OPDStream` backwards a whole trajectory at its close; the teacher
  scores are either given or computed by an optional teacher model, which may
  live on a second GPU and run concurrently.

Semantics follow reference src/thundersync/opd/objectives.py:93-1318.
"""

from __future__ import annotations

import concurrent.futures
from typing import Any

import torch

from thundersync_b200.engine.layers import Executor, Segment
from thundersync_b200.ops.logprob import lm_head_logprob

__all__ = ["OPDStream", "OPDTurnStream", "teacher_logprobs"]

_NORMALIZATIONS = ("token_mean", "sum")


class _StreamAdapter:
    """Forwards the event API to the run (objectives read the run's public API only)."""

    def __init__(self, run) -> None:
        self.run = run

    def open_group(self, group_id: int, prompt_tokens: list[int]) -> None:
        self.run.open_group(group_id, prompt_tokens)

    def open_groups_shared_prefix(self, prompts, **_kw) -> None:
        self.run.open_groups_shared_prefix(prompts)

    def append_turn(self, group_id: int, traj_id: int, tokens: list[int], scored: list[bool]) -> None:
        self.append_turns([(group_id, traj_id, tokens, scored)])

    def append_turns(self, items) -> None:
        self.run.append_turns(items)


class _ImmediateBackward(_StreamAdapter):
    def __init__(self, run, model: torch.nn.Module) -> None:
        if not run.boundary_cut:
            raise ValueError(
                f"{type(self).__name__} requires StreamingRun(boundary_cut=True): per-trajectory backwards "
                "through an uncut shared prompt would free it under the group's other trajectories"
            )
        super().__init__(run)
        self.params = [p for p in model.parameters() if p.requires_grad]
        if any(p.grad is not None for p in self.params):
            raise ValueError(f"{type(self).__name__} requires an empty parameter-gradient accumulator")
        self._versions = [p._version for p in self.params]
        self._closed: dict[int, set[int]] = {}
        self._finalized = False
        # every backward deposits into one fp32 buffer in the parameter-arena layout (bf16 parameters
        # would otherwise sum hundreds of per-action gradients in bf16 .grad tensors)
        self.arena = getattr(run, "arena", None)
        self._main: torch.Tensor | None = None

    def _sink(self):
        if self.arena is None:
            return None
        from thundersync_b200.ops.sink import GradSink

        if self._main is None:
            self._main = self.arena.new_buffer(torch.float32)
        return GradSink(self.arena, self._main)

    def use_main_grad_buffer(self, buf: torch.Tensor) -> None:
        """Accumulate into ``buf`` (fp32, arena layout, zeroed here), e.g. a data-parallel peer buffer."""
        if self.arena is None or buf.dtype != torch.float32 or buf.numel() < self.arena.numel:
            raise ValueError("the main gradient buffer must be fp32 and cover the parameter arena")
        buf.zero_()
        self._main = buf[: self.arena.numel]

    def main_grad(self) -> torch.Tensor | None:
        """The flat fp32 gradient (arena layout); normalised once the step is safe."""
        return self._main

    def _check_versions(self) -> None:
        if any(p._version != v for p, v in zip(self.params, self._versions)):
            raise RuntimeError("parameters changed inside a logical batch (version guard)")

    def append_turns(self, items) -> None:
        for gid, tid, _, _ in items:
            if tid in self._closed.get(gid, set()):
                raise RuntimeError(f"trajectory {tid} already closed")
        super().append_turns(items)

    def _register_close(self, traj_id: int) -> int:
        self._check_versions()
        gid = self.run.group_of(traj_id)
        closed = self._closed.setdefault(gid, set())
        if traj_id in closed:
            raise RuntimeError(f"trajectory {traj_id} already closed")
        closed.add(traj_id)
        return gid

    def close_group(self, group_id: int) -> None:
        self._check_versions()
        closed = self._closed.get(group_id, set())
        open_t = [t for t in self.run.trajectories_of(group_id) if t not in closed]
        if open_t:
            raise RuntimeError(f"group {group_id}: trajectories {open_t} not closed")
        self._closed.pop(group_id, None)
        self.run.finalize_group_boundary(group_id, sink=self._sink())
        self.run.free_group(group_id)

    @property
    def open_groups(self) -> list[int]:
        return sorted(self.run.open_group_ids())

    def assert_safe_to_step(self) -> None:
        self._check_versions()
        if self.open_groups:
            raise RuntimeError(
                f"optimizer step with open groups {self.open_groups}: their retained graphs reference "
                "current parameter values"
            )
        self.run.finalize_shared_prefixes(sink=self._sink())
        self.run.materialize_parameter_adjoints()


class _TokenLoss:
    """Shared loss arithmetic and batch normalisation bookkeeping."""

    def _init_loss(self, normalization: str) -> None:
        if normalization not in _NORMALIZATIONS:
            raise ValueError(f"OPD normalization must be 'token_mean' or 'sum', got {normalization!r}")
        self.normalization = normalization
        self._mass = 0.0
        self._numerator_dev: torch.Tensor | None = None
        self._numerator = 0.0
        self._finite: dict[torch.device, torch.Tensor] = {}

    @staticmethod
    def _check_inputs(scored_count: int, teacher: torch.Tensor, weights: torch.Tensor | None) -> None:
        if tuple(teacher.shape) != (scored_count,):
            raise ValueError(f"teacher logprobs have shape {tuple(teacher.shape)}, expected ({scored_count},)")
        if weights is not None:
            if weights.requires_grad:
                raise ValueError("OPD token_weights must be detached")
            if tuple(weights.shape) != (scored_count,):
                raise ValueError("token_weights must have one entry per scored token")
            if not bool(torch.isfinite(weights).all()) or bool((weights < 0).any()):
                raise ValueError("OPD token_weights must be finite and non-negative")

    def _note_finite(self, teacher: torch.Tensor) -> None:
        if teacher.device.type == "cpu":
            if not bool(torch.isfinite(teacher).all()):
                raise ValueError("teacher logprobs must be finite")
            return
        f = torch.isfinite(teacher).all()
        prev = self._finite.get(f.device)
        self._finite[f.device] = f if prev is None else prev & f

    @staticmethod
    def _loss(lp: torch.Tensor, old: torch.Tensor, teacher: torch.Tensor, weights: torch.Tensor | None):
        teacher = teacher.detach().to(device=lp.device, dtype=lp.dtype)
        ratio = torch.exp(lp - old)
        score = (old - teacher).detach()
        term = ratio * score
        if weights is not None:
            term = term * weights.detach().to(device=lp.device, dtype=lp.dtype)
        return term.sum()

    def _record(self, loss: torch.Tensor, n: int, weights: torch.Tensor | None, return_loss: bool):
        d = loss.detach().to(torch.float64)
        self._numerator_dev = d.clone() if self._numerator_dev is None else self._numerator_dev.add_(d)
        self._mass += n if weights is None else float(weights.detach().double().sum())
        return float(loss.detach()) if return_loss else None

    def _finalize_normalization(self, params: list[torch.Tensor], *, materialize: bool = True) -> None:
        for flag in self._finite.values():
            if not bool(flag):
                raise ValueError("teacher logprobs must be finite")
        div = self.normalization_divisor
        main = getattr(self, "_main", None)
        with torch.no_grad():
            if main is not None:
                if div != 1.0:
                    from thundersync_b200.ops.fold import scale_

                    scale_(main, 1.0 / div)
                if materialize:
                    for p in params:
                        v = self.arena.view(main, p)
                        if p.grad is None:
                            p.grad = v.to(p.dtype, copy=True)
                        else:
                            p.grad.add_(v.to(p.grad.dtype))
            if div != 1.0:
                # contributions that reached .grad outside the sink (parameters the arena does not hold)
                for p in params:
                    if p.grad is not None and (main is None or not materialize):
                        p.grad.div_(div)
        if self._numerator_dev is not None:
            self._numerator = float(self._numerator_dev)
            self._numerator_dev = None

    @property
    def normalization_divisor(self) -> float:
        return 1.0 if self.normalization == "sum" else max(self._mass, 1.0)

    @property
    def loss_value(self) -> float:
        if not self._finalized:
            raise RuntimeError("OPD loss_value requires assert_safe_to_step first")
        return self._numerator / self.normalization_divisor


class OPDTurnStream(_TokenLoss, _ImmediateBackward):
    """Backward each turn at teacher-score arrival; replay state adjoints at close."""

    def __init__(self, run, model: torch.nn.Module, *, normalization: str = "token_mean") -> None:
        if not run.turn_boundary_rebuild:
            raise ValueError("OPDTurnStream requires StreamingRun(turn_boundary_rebuild=True)")
        _ImmediateBackward.__init__(self, run, model)
        self._init_loss(normalization)
        # a turn without a scored token has no loss: it forwards only when a later turn of its trajectory
        # needs its state, and a trailing one never does
        run.defer_unscored_turns = True

    def append_scored_turn(self, group_id, traj_id, tokens, scored, *, teacher_logprobs, token_weights=None,
                           return_loss: bool = True):
        return self.append_scored_turns([(group_id, traj_id, tokens, scored, teacher_logprobs, token_weights)],
                                        return_loss=return_loss)[0]

    def append_scored_turns(self, items, *, return_loss: bool = True) -> list[float | None]:
        if not items:
            raise ValueError("append_scored_turns needs at least one item")
        if self._finalized:
            raise RuntimeError("cannot append a turn after OPD finalization")
        self._check_versions()
        seen = set()
        for gid, tid, tokens, scored, teacher, weights in items:
            if tid in seen:
                raise ValueError(f"trajectory {tid} appears twice in one scored-turn pack")
            seen.add(tid)
            if tid in self._closed.get(gid, set()):
                raise RuntimeError(f"trajectory {tid} already closed")
            self._check_inputs(sum(bool(s) for s in scored), teacher, weights)
        for *_, teacher, _w in items:
            self._note_finite(teacher)
        self.run.append_turns([(g, t, tk, sc) for g, t, tk, sc, _, _ in items], joint_backward=True)
        losses, meta = [], []
        for gid, tid, tokens, scored, teacher, weights in items:
            lp, old = self.run.consume_latest_turn_logprobs(tid)
            if lp.numel() == 0:
                meta.append(None)
                continue
            if not torch.equal(lp.detach(), old):
                raise RuntimeError("OPD requires on-policy behavior logprobs from the same turn")
            loss = self._loss(lp, old, teacher, weights)
            losses.append(loss)
            meta.append((loss, lp.numel(), weights))
        if losses:
            src = ("trajectory_turn_pack", tuple(t for _, t, *_ in items))
            self.run.backward_with_boundary_adjoint_capture(losses, source=src, sink=self._sink())
        return [None if m is None else self._record(m[0], m[1], m[2], return_loss) for m in meta]

    def close_trajectory(self, traj_id: int) -> None:
        self.close_trajectories([traj_id])

    def close_trajectories(self, traj_ids: list[int]) -> None:
        if self._finalized:
            raise RuntimeError("cannot close a trajectory after OPD finalization")
        if len(set(traj_ids)) != len(traj_ids):
            raise ValueError("a trajectory appears twice in one closure cohort")
        for t in traj_ids:
            self._register_close(t)
        self.run.finalize_trajectories_turn_boundaries(list(traj_ids), sink=self._sink())
        for t in traj_ids:
            self.run.free_trajectory(t)

    def assert_safe_to_step(self, *, materialize: bool = True) -> None:
        if self._finalized:
            return
        _ImmediateBackward.assert_safe_to_step(self)
        self._finalize_normalization(self.params, materialize=materialize)
        self._finalized = True


def teacher_logprobs(teacher: torch.nn.Module, prompt: list[int], turns: list[tuple[list[int], list[bool]]],
                     *, device: torch.device | None = None) -> torch.Tensor:
    """The frozen teacher's fp32 log-probs of every scored turn token (no graph)."""
    dev = device or next(teacher.parameters()).device
    toks = list(prompt) + [t for tk, _ in turns for t in tk]
    scored = [False] * len(prompt) + [bool(s) for _, sc in turns for s in sc]
    ids = torch.tensor(toks, device=dev)
    pos = torch.arange(len(toks), device=dev)
    with torch.no_grad():
        ex = Executor(teacher)
        h, _ = ex.run(ids, pos, [Segment(0, len(toks), [])])
        idx = [i for i, s in enumerate(scored) if s and i > 0]
        if not idx:
            return torch.zeros(0, dtype=torch.float32, device=dev)
        src = torch.tensor([i - 1 for i in idx], device=dev)
        tgt = torch.tensor([toks[i] for i in idx], device=dev)
        return lm_head_logprob(h.index_select(0, src), ex.head_weight(), tgt)


class OPDStream(_TokenLoss, _ImmediateBackward):
    """Trajectory-close OPD: one backward per trajectory when it closes.

    ``teacher``: an optional frozen model that scores closed trajectories
    itself; with ``concurrent_teacher_replay`` it runs on its own device in a
    worker thread while the student differentiates the previous trajectory.
    A teacher failure poisons the step (``assert_safe_to_step`` re-raises).
    ``joint_backward``: the trajectories closed by one call run one backward over
    their summed losses. ``closure_cohort_vjp`` and ``ragged_cohort_attention``
    are accepted for the reference's signature and change nothing here: a
    closure cohort's one backward is ``joint_backward``'s, and segments of a
    pack always attend through the packed attention kernels.
    """

    def __init__(self, run, model: torch.nn.Module, *, teacher: torch.nn.Module | None = None,
                 normalization: str = "token_mean", joint_backward: bool = False, closure_cohort_vjp: Any = None,
                 ragged_cohort_attention: bool = False, concurrent_teacher_replay: bool = False) -> None:
        _ImmediateBackward.__init__(self, run, model)
        self._init_loss(normalization)
        self.teacher = teacher
        if teacher is not None:
            for p in teacher.parameters():
                p.requires_grad_(False)
        self.concurrent = bool(concurrent_teacher_replay)
        if self.concurrent and teacher is None:
            raise ValueError("concurrent_teacher_replay needs a teacher model")
        self._pool = concurrent.futures.ThreadPoolExecutor(1) if self.concurrent else None
        self._poison: BaseException | None = None
        self._prompts: dict[int, list[int]] = {}
        # several trajectories closed in one call run one backward over their summed losses
        self.joint_backward = bool(joint_backward)

    def open_group(self, group_id: int, prompt_tokens: list[int]) -> None:
        self._prompts[group_id] = list(prompt_tokens)
        super().open_group(group_id, prompt_tokens)

    def _teacher_scores(self, traj_id: int):
        gid = self.run.group_of(traj_id)
        turns = self.run._trajs[traj_id].turns
        return teacher_logprobs(self.teacher, self._prompts[gid], turns)

    def close_trajectory(self, traj_id: int, *, teacher_logprobs: torch.Tensor | None = None,
                         token_weights: torch.Tensor | None = None) -> None:
        self.close_trajectories([(traj_id, teacher_logprobs, token_weights)])

    def close_trajectories(self, items) -> None:
        if self._finalized:
            raise RuntimeError("cannot close a trajectory after OPD finalization")
        if self._poison is not None:
            raise RuntimeError("a concurrent teacher replay failed; this step is poisoned") from self._poison
        norm = [(i, None, None) if isinstance(i, int) else (i[0], i[1] if len(i) > 1 else None,
                                                             i[2] if len(i) > 2 else None) for i in items]
        joint = self.joint_backward and len(norm) > 1
        losses: list[tuple[torch.Tensor, int, Any]] = []
        futures = {}
        for tid, teacher, _ in norm:
            if teacher is None:
                if self.teacher is None:
                    raise ValueError(f"trajectory {tid} closed without teacher logprobs and no teacher model")
                if self._pool is not None:
                    futures[tid] = self._pool.submit(self._teacher_scores, tid)
        for tid, teacher, weights in norm:
            self._register_close(tid)
            lp = self.run.logprobs(tid)
            old = self.run.old_logprobs(tid)
            if teacher is None:
                try:
                    teacher = futures[tid].result() if tid in futures else self._teacher_scores(tid)
                except BaseException as exc:
                    self._poison = exc
                    raise
            self._check_inputs(lp.numel(), teacher, weights)
            self._note_finite(teacher)
            if lp.numel():
                loss = self._loss(lp, old, teacher, weights)
                if joint:
                    losses.append((loss, lp.numel(), weights))
                    continue
                self.run.backward_with_boundary_adjoint_capture(loss, source=("trajectory", tid), sink=self._sink())
                self._record(loss, lp.numel(), weights, False)
            if not joint:
                self.run.free_trajectory(tid)
        if joint:
            if losses:
                self.run.backward_with_boundary_adjoint_capture(
                    [x for x, _, _ in losses], source=("trajectory_cohort", tuple(t for t, _, _ in norm)),
                    sink=self._sink())
                for loss, n, weights in losses:
                    self._record(loss, n, weights, False)
            for tid, _, _ in norm:
                self.run.free_trajectory(tid)

    def assert_safe_to_step(self, *, materialize: bool = True) -> None:
        if self._poison is not None:
            raise RuntimeError("a concurrent teacher replay failed; this step is poisoned") from self._poison
        if self._finalized:
            return
        _ImmediateBackward.assert_safe_to_step(self)
        self._finalize_normalization(self.params, materialize=materialize)
        self._finalized = True
        if self._pool is not None:
            self._pool.shutdown(wait=True)
