"""RewardLinearBackward: per-trajectory GRPO backward at reward arrival (C30).

GRPO's update is ``Σ_i A_i ∇S_i`` with ``S_i = Σ_t w_t log π(y_t | ctx)``
and the group-normalised advantage ``A_i = (r_i − μ)/(σ + ε)`` (population
std, float64 moments in trajectory order). ``μ`` and ``σ`` are unknown until
the group's last reward lands, so each trajectory's gradient is folded into
two per-group statistics when it is computed,

    G2 = Σ_i ∇S_i,   G1 = Σ_i r_i ∇S_i,

and the group close is one fused AXPY: ``grad += (G1 − μ·G2)/σ``
(reference: src/thundersync/grpo/reward_linear.py:256-3718). The prompt's
boundary adjoints are folded the same way and the prompt is backwarded once
with ``(B1 − μ·B2)/σ``.

B200-first execution:

* statistics are flat fp32 buffers in the parameter-arena layout, resident on
  the device by default (``source_offload_mode="device_resident"``) or on the
  host (the reference default, ``source_offload_device="cpu"``);
* a trajectory's weight gradients go straight from the GEMMs into a gradient
  sink: with binary rewards (``configure_binary_rewards``) the sink *is* the
  group's P (r = 1) or N (r = 0) statistic, so no per-trajectory gradient
  exists at all; otherwise one fp32 scratch receives it and one fused kernel
  folds it into G1/G2;
* when every reward of the group is already known (``direct_when_group_bound``)
  the trajectory backwards with its advantage as the sink scale straight into
  the batch gradient.
"""

from __future__ import annotations

import contextlib

import logging
import math
import time
from dataclasses import dataclass, field
from typing import Any, Callable

import torch

from thundersync_b200.grpo.config import DEFAULT_GRPO_EPSILON, SOURCE_OFFLOAD_MODES, SOURCE_REDUCTION_MODES
from thundersync_b200.ops.fold import axpby_, fold_
from thundersync_b200.ops.sink import GradSink

log = logging.getLogger(__name__)

__all__ = ["RewardLinearBackward"]


@dataclass
class _GroupAccum:
    gid: int
    traj_ids: list[int]
    rewards: dict[int, float] = field(default_factory=dict)
    closed: set[int] = field(default_factory=set)
    folded: list[int] = field(default_factory=list)  # readiness order
    g1: torch.Tensor | None = None  # or P in binary mode
    g2: torch.Tensor | None = None  # or N in binary mode
    b1: list[torch.Tensor | None] = field(default_factory=list)
    b2: list[torch.Tensor | None] = field(default_factory=list)
    slot: Any = None  # device statistic home, when the pool had one
    direct: bool = False
    direct_boundary: list[torch.Tensor | None] = field(default_factory=list)
    prepared: dict[int, Any] = field(default_factory=dict)
    close_requested: bool = False
    done: bool = False


class RewardLinearBackward:
    """Streams per-trajectory backwards; the group barrier becomes an AXPY."""

    def __init__(
        self,
        run,
        model: torch.nn.Module,
        *,
        eps: float = DEFAULT_GRPO_EPSILON,
        source_offload_device: str | torch.device | None = "cpu",
        source_offload_mode: str = "blocking",
        source_reduction_mode: str = "unrestricted_statistics",
        source_reduction_pack_size: int = 1,
        source_offload_pinned_windows: int = 2,
        statistic_device: str | torch.device | None = None,
        device_statistic_slots: int | None = None,
        statistic_keep_source_dtype: bool = False,
        source_reduction_worker_count: int = 2,
        source_offload_worker_count: int = 2,
        source_offload_window_bytes: int = 256 * 1024 * 1024,
        source_offload_hbm_threshold: float = 0.65,
        source_spill_directory: Any = None,
        source_pinned_arena: Any = None,
        defer_group_close: bool = False,
        source_copy_during_backward: bool = False,
        source_release_during_backward: bool = False,
        combine_known_reward_sources: bool = False,
        direct_when_group_bound: bool = False,
    ) -> None:
        if not run.boundary_cut:
            raise ValueError(
                "RewardLinearBackward requires StreamingRun(boundary_cut=True); without the "
                "cut each trajectory backward re-traverses the shared prompt"
            )
        if source_offload_mode not in SOURCE_OFFLOAD_MODES:
            raise ValueError(f"source_offload_mode must be one of {SOURCE_OFFLOAD_MODES}")
        if source_reduction_mode not in SOURCE_REDUCTION_MODES:
            raise ValueError(f"source_reduction_mode must be one of {SOURCE_REDUCTION_MODES}")
        if source_reduction_pack_size < 1:
            raise ValueError("source_reduction_pack_size must be positive")
        if not eps > 0:
            raise ValueError("eps must be positive")
        if run.arena is None:
            raise ValueError("RewardLinearBackward needs every trainable parameter on one device and dtype")
        self.run = run
        self.model = model
        self.eps = float(eps)
        self.arena = run.arena
        self.source_offload_mode = source_offload_mode
        if source_offload_device in ("none",):
            source_offload_device = None
        if statistic_device is not None:
            stat_dev = torch.device(statistic_device)
        elif source_offload_mode == "device_resident" or source_offload_device is None:
            stat_dev = run.device
        else:
            stat_dev = torch.device(source_offload_device)
        self.statistic_device = stat_dev
        if source_copy_during_backward or source_release_during_backward:
            from thundersync_b200.config import ConfigError

            raise ConfigError("copying or releasing a source's parameter gradients during its backward is not "
                              "built here: a source goes from the GEMM epilogues into one fp32 buffer and is "
                              "folded once (set source_copy_during_backward / source_release_during_backward "
                              "to False)")
        if not 0.0 < source_offload_hbm_threshold <= 1.0:
            raise ValueError("source_offload_hbm_threshold must be in (0, 1]")
        for name, value in (("source_offload_pinned_windows", source_offload_pinned_windows),
                            ("source_offload_worker_count", source_offload_worker_count),
                            ("source_reduction_worker_count", source_reduction_worker_count)):
            if value < 1:
                raise ValueError(f"{name} must be positive")
        if source_offload_window_bytes < 4096:
            raise ValueError("source_offload_window_bytes must be at least 4096")
        # host statistics: streamed through page-locked windows (grpo/host_fold.py)
        self._host_fold_options = dict(window_bytes=int(source_offload_window_bytes),
                                       windows=int(source_offload_pinned_windows),
                                       offload_workers=int(source_offload_worker_count),
                                       reduction_workers=int(source_reduction_worker_count),
                                       arena=source_pinned_arena)
        self._host_fold = None
        self._spill_dir = source_spill_directory
        self._hbm_threshold = float(source_offload_hbm_threshold)
        self._keep_source_dtype = bool(statistic_keep_source_dtype)
        self.direct_when_group_bound = direct_when_group_bound
        self.combine_known_reward_sources = combine_known_reward_sources
        self.defer_group_close = defer_group_close
        self._binary = False
        self._stat_slots = int(device_statistic_slots or 0)
        from thundersync_b200.grpo.close_profiler import ClosePackProfiler

        self._close_profiler = ClosePackProfiler.from_env()
        self._profile_rank = int(__import__("os").environ.get("RANK", "0"))
        self._profile_step = 0
        self._stat_pool = None
        self._groups: dict[int, _GroupAccum] = {}
        self._traj_group: dict[int, int] = {}
        self._main: torch.Tensor | None = None
        self._scratch: torch.Tensor | None = None
        self._aborted = False
        self._stepped = False
        self._branch_observer: Callable | None = None
        self._scope: dict[str, Any] = {}
        self._report = {
            "sources": 0, "direct_sources": 0, "binary_sources": 0, "folds": 0,
            "group_closes": 0, "uniform_reward_groups": 0, "fold_s": 0.0, "backward_s": 0.0,
            "statistic_device": str(stat_dev), "device_groups_below_hbm_threshold": 0, "host_groups": 0,
            "combined_sources": 0, "group_closes_deferred": 0,
        }
        # group closes requested while host folds were still running (defer_group_close); they run in
        # request order at later safe points
        self._requested_closes: list[int] = []
        self._versions = {id(p): p._version for p in run._trainable}

    # ------------------------------------------------------------ configuration
    def configure_binary_rewards(self) -> None:
        """Rewards are in {0, 1}: keep P = Σ_{r=1}∇S and N = Σ_{r=0}∇S instead of G1/G2."""
        if any(acc.g2 is not None for acc in self._groups.values()):
            raise RuntimeError("binary rewards must be configured before the first source folds")
        self._binary = True

    def set_statistics_branch_observer(self, observer: Callable | None) -> None:
        self._branch_observer = observer

    def set_diagnostic_scope(self, **scope: Any) -> None:
        self._scope.update(scope)
        if "rank" in scope:
            self._profile_rank = int(scope["rank"])
        if "step" in scope:
            self._profile_step = int(scope["step"])

    # ------------------------------------------------------------ buffers
    def _pipeline(self):
        if self._host_fold is None:
            from thundersync_b200.grpo.host_fold import HostFoldPipeline

            self._host_fold = HostFoldPipeline.shared(self.run.device, **self._host_fold_options)
        return self._host_fold

    def _main_grad(self) -> torch.Tensor:
        if self._main is None:
            self._main = self.arena.new_buffer(torch.float32)
        return self._main

    def use_main_grad_buffer(self, buf: torch.Tensor) -> None:
        """Accumulate the batch gradient into ``buf`` (fp32, arena layout, zeroed here).

        The data-parallel trainer passes a peer-mapped buffer so the step's
        reduction reads and writes it in place over NVLink.
        """
        if buf.dtype != torch.float32 or buf.numel() < self.arena.numel:
            raise ValueError("the main gradient buffer must be fp32 and cover the arena")
        buf.zero_()
        self._main = buf[: self.arena.numel]

    def main_grad(self) -> torch.Tensor | None:
        """The flat fp32 batch gradient (arena layout); None before any close."""
        return self._main

    def _stat(self, device: torch.device | None = None) -> torch.Tensor:
        device = self.statistic_device if device is None else device
        if device.type == "cpu":
            from thundersync_b200.grpo.host_fold import host_statistic

            dtype = self.arena.dtype if self._keep_source_dtype else torch.float32
            return host_statistic(self.arena.numel, dtype, self._spill_dir)
        return torch.zeros(self.arena.numel, dtype=torch.float32, device=device)

    def _device_has_room(self) -> bool:
        """Blocking sources: a group's statistics stay on the device while the device's reserved memory,
        plus the pair, stays below ``source_offload_hbm_threshold`` of its capacity."""
        dev = self.run.device
        if self.source_offload_mode != "blocking" or dev.type != "cuda":
            return False
        free, total = torch.cuda.mem_get_info(dev)
        pair = 2 * 4 * self.arena.numel
        used = total - free
        return used + pair <= self._hbm_threshold * total

    def _stat_pair(self, acc) -> tuple[torch.Tensor, torch.Tensor]:
        """(reward-weighted, unit) statistics of a group: a preallocated device home when one is free."""
        if self.statistic_device.type == "cpu" and self._device_has_room():
            self._report["device_groups_below_hbm_threshold"] += 1
            return self._stat(self.run.device), self._stat(self.run.device)
        if self.statistic_device.type == "cpu":
            self._report["host_groups"] += 1
        if self._stat_slots and self.statistic_device.type == "cuda":
            if self._stat_pool is None:
                from thundersync_b200.grpo.device_statistics import DeviceStatisticPool

                self._stat_pool = DeviceStatisticPool(self.arena.numel, torch.float32, slots=self._stat_slots,
                                                      device=self.statistic_device)
            slot = self._stat_pool.acquire(acc.gid)
            if slot is not None:
                acc.slot = slot
                return slot.reward, slot.unit
        return self._stat(), self._stat()

    def _drop_stats(self, acc) -> None:
        acc.g1 = acc.g2 = None
        if acc.slot is not None:
            self._stat_pool.release(acc.slot)
            acc.slot = None

    # ------------------------------------------------------------ groups
    def open_group(self, group_id: int, prompt: list[int], traj_ids: list[int]) -> None:
        self.run.open_group(group_id, prompt)
        self.register_group_trajectories(group_id, traj_ids)

    def register_group_trajectories(self, group_id: int, traj_ids: list[int]) -> None:
        if group_id in self._groups:
            raise ValueError(f"group {group_id} is already registered")
        ids = [int(t) for t in traj_ids]
        if len(set(ids)) != len(ids) or not ids:
            raise ValueError("a group needs distinct trajectory ids")
        for t in ids:
            if t in self._traj_group:
                raise ValueError(f"trajectory {t} is already registered")
            self._traj_group[t] = group_id
        self._groups[group_id] = _GroupAccum(group_id, ids)

    def open_groups(self) -> list[int]:
        return [g for g, a in self._groups.items() if not a.done]

    def group_fully_bound(self, group_id: int) -> bool:
        acc = self._groups[group_id]
        return all(t in acc.rewards for t in acc.traj_ids)

    def registered_groups_fully_bound(self) -> bool:
        return all(self.group_fully_bound(g) for g, a in self._groups.items() if not a.done)

    def known_slab_capacity(self) -> int | None:
        """Free slabs a known close could take beyond the held-source budget; None: unbounded here (a
        known close differentiates into one reused scratch buffer and folds at once, holding nothing)."""
        return None

    # ------------------------------------------------------------ trajectory events
    def close_trajectory(self, traj_id: int, reward: float, token_weights: torch.Tensor | None = None) -> None:
        self.close_trajectories([(traj_id, reward, token_weights)])

    def close_trajectories(self, items: list) -> None:
        """Content complete and reward landed: differentiate, then fold."""
        norm = []
        for item in items:
            tid, reward = item[0], item[1]
            w = item[2] if len(item) > 2 else None
            if reward is None or not math.isfinite(float(reward)):
                raise ValueError(f"trajectory {tid} closed without a finite reward")
            norm.append((int(tid), float(reward), w))
        prof = self._close_profiler
        window = contextlib.nullcontext()
        if prof is not None:
            window = prof.capture(rank=self._profile_rank, step=self._profile_step,
                                  trajectory_ids=[t for t, _, _ in norm],
                                  branch_tokens=[self.run.trajectory_tokens(t) for t, _, _ in norm])
        with window:
            for tid, reward, _ in norm:
                self._record(tid, reward)
            for cohort in self._cohorts(norm):
                if len(cohort) > 1:
                    self._differentiate_cohort([t for t, _, _ in cohort], cohort[0][1])
                else:
                    tid, reward, w = cohort[0]
                    self._differentiate(tid, reward, w)
        self._run_requested_closes(wait=False)

    def _cohorts(self, items: list[tuple[int, float, Any]]) -> list[list[tuple[int, float, Any]]]:
        """With ``combine_known_reward_sources``: closes of one group that share a reward (and carry no
        token weights) run as one source -- one packed rebuild, one backward, one fold -- since the
        statistics only ever see ``r·Σ∇S`` and ``Σ∇S`` of them. Otherwise one cohort per close."""
        if not self.combine_known_reward_sources or len(items) < 2:
            return [[it] for it in items]
        out: list[list[tuple[int, float, Any]]] = []
        index: dict[tuple[int, float], int] = {}
        for it in items:
            tid, reward, w = it
            acc = self._acc(tid)
            direct = acc.direct or (self.direct_when_group_bound and self.group_fully_bound(acc.gid))
            if w is not None or direct or tid in acc.closed:
                out.append([it])
                continue
            key = (acc.gid, reward)
            if key in index:
                out[index[key]].append(it)
            else:
                index[key] = len(out)
                out.append([it])
        return out

    def _differentiate_cohort(self, tids: list[int], reward: float) -> None:
        acc = self._acc(tids[0])
        self._check_versions()
        t0 = time.perf_counter()
        if self.run.stream_turns:
            lps = [self._logprobs(t) for t in tids]
        else:
            lps = self.run.rebuild_logprobs(tids, joint_backward=True)  # one packed forward, one backward
        s = torch.cat([lp.reshape(-1) for lp in lps]).sum()
        binary_sink = self._binary and self.statistic_device == self.run.device
        if binary_sink:
            if acc.g2 is None:
                acc.g1, acc.g2 = self._stat_pair(acc)
            sink = GradSink(self.arena, acc.g1 if reward == 1.0 else acc.g2)
        else:
            if self._scratch is None or self._scratch.device != self.run.device:
                self._scratch = self.arena.new_buffer(torch.float32)
            else:
                self._scratch.zero_()
            sink = GradSink(self.arena, self._scratch)
        if s.requires_grad:
            self.run.backward_with_boundary_adjoint_capture(s, source=("cohort", tuple(tids)), sink=sink)
        bnd = self.run.boundary(acc.gid).drain()
        for t in tids:
            self.run.free_trajectory(t)
        self._report["backward_s"] += time.perf_counter() - t0
        self._report["sources"] += 1
        self._report["combined_sources"] += len(tids)
        if binary_sink:
            self._fold_boundary(acc, reward, bnd)
            acc.folded.extend(tids)
            self._report["binary_sources"] += 1
        else:
            self._fold(acc, tids[0], reward, self._scratch, bnd)
            acc.folded.extend(tids[1:])
        acc.closed.update(tids)

    def prepare_trajectory(self, traj_id: int, token_weights=None) -> None:
        self.prepare_trajectories([(traj_id, token_weights)] if token_weights is not None else [traj_id])

    def prepare_trajectories(self, items: list) -> None:
        """Content complete, reward unknown: compute and hold the source."""
        for item in items:
            tid, w = (item, None) if not isinstance(item, tuple) else (item[0], item[1] if len(item) > 1 else None)
            tid = int(tid)
            acc = self._acc(tid)
            if tid in acc.prepared or tid in acc.closed:
                raise ValueError(f"trajectory {tid} was already prepared or closed")
            if tid in acc.rewards:
                self._differentiate(tid, acc.rewards[tid], w)
                continue
            src = self.arena.new_buffer(torch.float32)
            bnd = self._backward_source(tid, w, GradSink(self.arena, src))
            acc.prepared[tid] = (src, bnd)
        self._run_requested_closes(wait=False)

    def bind_reward(self, traj_id: int, reward: float) -> None:
        self.bind_rewards([(traj_id, reward)])

    def bind_rewards(self, binds: list[tuple[int, float]]) -> None:
        for tid, reward in binds:
            if reward is None or not math.isfinite(float(reward)):
                raise ValueError(f"trajectory {tid} bound without a finite reward")
        for tid, reward in binds:
            tid, reward = int(tid), float(reward)
            acc = self._acc(tid)
            self._record(tid, reward)
            if tid in acc.prepared:
                src, bnd = acc.prepared.pop(tid)
                self._fold(acc, tid, reward, src, bnd)
                acc.closed.add(tid)
        self._run_requested_closes(wait=False)

    def record_rewards(self, items: list[tuple[int, float]]) -> None:
        for tid, reward in items:
            self._record(int(tid), float(reward))

    def _record(self, tid: int, reward: float) -> None:
        acc = self._acc(tid)
        if self._binary and reward not in (0.0, 1.0):
            raise ValueError(f"binary rewards must be 0 or 1, got {reward}")
        prev = acc.rewards.get(tid)
        if prev is not None and prev != reward:
            raise ValueError(f"trajectory {tid} already has reward {prev}")
        acc.rewards[tid] = reward

    def _acc(self, tid: int) -> _GroupAccum:
        gid = self._traj_group.get(tid)
        if gid is None:
            raise KeyError(f"trajectory {tid} is not registered with any group")
        acc = self._groups[gid]
        if acc.done:
            raise RuntimeError(f"group {gid} is already closed")
        return acc

    # ------------------------------------------------------------ differentiation
    def _logprobs(self, tid: int) -> torch.Tensor:
        run = self.run
        if run.stream_turns:
            t = run._trajs[tid]
            if t.forwarded_turns < len(t.turns):
                run.forward_deferred_turns(tid)
            return run.logprobs(tid)
        return run.rebuild_logprobs([tid])[0]

    def _objective(self, lp: torch.Tensor, w) -> torch.Tensor:
        if w is None:
            return lp.sum()
        w = torch.as_tensor(w, dtype=lp.dtype, device=lp.device)
        if w.shape != lp.shape:
            raise ValueError(f"token_weights shape {tuple(w.shape)} != scored tokens {tuple(lp.shape)}")
        return (lp * w).sum()

    def _backward_source(self, tid: int, w, sink: GradSink) -> list[torch.Tensor | None]:
        """Backward one trajectory into ``sink``; returns its boundary adjoint."""
        self._check_versions()
        t0 = time.perf_counter()
        lp = self._logprobs(tid)
        s = self._objective(lp, w)
        gid = self._traj_group[tid]
        if s.requires_grad:
            self.run.backward_with_boundary_adjoint_capture(s, source=("trajectory", tid), sink=sink)
        bnd = self.run.boundary(gid).drain()
        self.run.free_trajectory(tid)
        self._report["backward_s"] += time.perf_counter() - t0
        self._report["sources"] += 1
        if self._branch_observer is not None:
            self._branch_observer(tid, sink.buffer)
        return bnd

    def _differentiate(self, tid: int, reward: float, w) -> None:
        acc = self._acc(tid)
        if tid in acc.closed:
            raise ValueError(f"trajectory {tid} is already closed")
        if (self.direct_when_group_bound and self.group_fully_bound(acc.gid)) or acc.direct:
            # Every reward of the group is known: A_i is final, so the source
            # goes straight into the batch gradient with A_i as the sink scale.
            mean, std = self._moments(acc)
            a = (reward - mean) / std
            acc.direct = True
            bnd = self._backward_source(tid, w, GradSink(self.arena, self._main_grad(), scale=a))
            self._add_direct_boundary(acc, bnd, a)
            acc.closed.add(tid)
            self._report["direct_sources"] += 1
            return
        if self._binary and self.statistic_device == self.run.device:
            # The sink is the statistic itself: P for r = 1, N for r = 0.
            if acc.g2 is None:
                acc.g1, acc.g2 = self._stat_pair(acc)
            target = acc.g1 if reward == 1.0 else acc.g2
            bnd = self._backward_source(tid, w, GradSink(self.arena, target))
            self._fold_boundary(acc, reward, bnd)
            acc.folded.append(tid)
            acc.closed.add(tid)
            self._report["binary_sources"] += 1
            return
        if self._scratch is None or self._scratch.device != self.run.device:
            self._scratch = self.arena.new_buffer(torch.float32)
        else:
            self._scratch.zero_()
        bnd = self._backward_source(tid, w, GradSink(self.arena, self._scratch))
        self._fold(acc, tid, reward, self._scratch, bnd)
        acc.closed.add(tid)

    def _fold(self, acc: _GroupAccum, tid: int, reward: float, src: torch.Tensor, bnd) -> None:
        t0 = time.perf_counter()
        if acc.g2 is None:
            acc.g1, acc.g2 = self._stat_pair(acc)
        if acc.g2.device.type == "cpu" and src.is_cuda:
            # host statistics: windowed device->host copies, host adds in the background
            pipe = self._pipeline()
            if self._binary:
                pipe.fold(src, None, acc.g1 if reward == 1.0 else acc.g2, 0.0)
            else:
                pipe.fold(src, acc.g1, acc.g2, reward)
        elif self._binary:
            (acc.g1 if reward == 1.0 else acc.g2).add_(src.to(acc.g2.device))
        else:
            fold_(acc.g1, acc.g2, src if src.device == acc.g2.device else src.to(acc.g2.device), reward)
        self._fold_boundary(acc, reward, bnd)
        acc.folded.append(tid)
        self._report["folds"] += 1
        self._report["fold_s"] += time.perf_counter() - t0

    def _fold_boundary(self, acc: _GroupAccum, reward: float, bnd: list[torch.Tensor | None]) -> None:
        if not acc.b1:
            acc.b1 = [None] * len(bnd)
            acc.b2 = [None] * len(bnd)
        for i, a in enumerate(bnd):
            if a is None:
                continue
            a = a.float()
            if self._binary:
                slot = acc.b1 if reward == 1.0 else acc.b2
                slot[i] = a if slot[i] is None else slot[i].add_(a)
            else:
                acc.b2[i] = a.clone() if acc.b2[i] is None else acc.b2[i].add_(a)
                if reward != 0.0:
                    acc.b1[i] = a * reward if acc.b1[i] is None else acc.b1[i].add_(a, alpha=reward)

    def _add_direct_boundary(self, acc: _GroupAccum, bnd, a: float) -> None:
        if not acc.direct_boundary:
            acc.direct_boundary = [None] * len(bnd)
        for i, x in enumerate(bnd):
            if x is None:
                continue
            x = x.float() * a
            acc.direct_boundary[i] = x if acc.direct_boundary[i] is None else acc.direct_boundary[i].add_(x)

    # ------------------------------------------------------------ close
    def _moments(self, acc: _GroupAccum) -> tuple[float, float]:
        r = torch.tensor([acc.rewards[t] for t in sorted(acc.rewards)], dtype=torch.float64)
        return float(r.mean()), float(r.std(unbiased=False)) + self.eps

    def final_advantage(self, traj_id: int) -> float:
        acc = self._acc(traj_id)
        if not self.group_fully_bound(acc.gid):
            raise RuntimeError("the group's rewards are not all known")
        mean, std = self._moments(acc)
        return (acc.rewards[traj_id] - mean) / std

    def wait_for_trajectory_reduction(self, group_id: int, trajectory_id: int) -> None:
        """Return once the trajectory's source is folded into its group's statistics: device folds are
        stream-ordered, host folds (statistics on the host) are waited for."""
        acc = self._groups[group_id]
        if int(trajectory_id) not in acc.traj_ids:
            raise KeyError(f"trajectory {trajectory_id} is not in group {group_id}")
        if self._host_fold is not None:
            self._host_fold.drain()

    def group_reduction_complete(self, group_id: int) -> bool:
        """No source of the group waits for its reward and no host fold is still running."""
        acc = self._groups[group_id]
        return not acc.prepared and not self._folds_pending()

    @property
    def pending_reduction_source_count(self) -> int:
        """Host folds still running (0 when statistics stay on the device)."""
        return 0 if self._host_fold is None else self._host_fold.pending_count()

    @property
    def held_source_count(self) -> int:
        return sum(len(a.prepared) for a in self._groups.values())

    def _folds_pending(self) -> bool:
        return self._host_fold is not None and self._host_fold.pending()

    def _run_requested_closes(self, *, wait: bool) -> None:
        """Run requested group closes in request order; without ``wait`` stop at the first one that
        would have to wait for host folds still running."""
        while self._requested_closes:
            if not wait and self._folds_pending():
                return
            self._close_group_now(self._requested_closes.pop(0))

    def close_group(self, group_id: int) -> None:
        """All rewards in: combine the statistics, backward the prompt once.

        With ``defer_group_close``, a close that would wait for host folds still running is recorded and
        the call returns; recorded closes run in request order (so the parameter gradient accumulates in
        the same order as closing at once) at the end of a later prepare, bind or close call, at the next
        ``close_group``, or in :meth:`assert_safe_to_step`, which waits for the folds (reference
        src/thundersync/grpo/reward_linear.py:3359-3400)."""
        acc = self._groups.get(group_id)
        if acc is None:
            raise KeyError(f"group {group_id} is not registered")
        if acc.done or group_id in self._requested_closes:
            raise RuntimeError(f"group {group_id} is already closed")
        missing = [t for t in acc.traj_ids if t not in acc.closed]
        if missing:
            raise RuntimeError(f"group {group_id} still has open trajectories {missing}")
        if self.defer_group_close:
            self._requested_closes.append(group_id)
            self._run_requested_closes(wait=False)
            if group_id in self._requested_closes:
                self._report["group_closes_deferred"] += 1
            return
        self._close_group_now(group_id)

    def _close_group_now(self, group_id: int) -> None:
        acc = self._groups[group_id]
        self._check_versions()
        mean, std = self._moments(acc)
        main = self._main_grad()
        rewards = {acc.rewards[t] for t in acc.traj_ids}
        uniform = len(rewards) == 1
        # uniform group: sum_i A_i g_i = A * G2 with the float64 A (exactly 0
        # when the mean equals the reward) instead of dividing the
        # statistics' rounding residual by eps
        a_uni = (next(iter(rewards)) - mean) / std if uniform else 0.0
        if uniform:
            self._report["uniform_reward_groups"] += 1
        adjoints: list[torch.Tensor | None] = []
        if acc.g2 is not None and acc.g2.device.type == "cpu" and main.is_cuda:
            # host statistics: combined on the host window by window and added on the device
            inv = 1.0 / std
            pipe = self._pipeline()
            if self._binary:
                a, b = (a_uni, a_uni) if uniform else ((1.0 - mean) * inv, -mean * inv)
                pipe.combine_into(main, acc.g1, acc.g2, a, b)
            elif uniform:
                pipe.combine_into(main, acc.g2, None, a_uni, 0.0)
            else:
                pipe.combine_into(main, acc.g1, acc.g2, inv, -mean * inv)
        elif acc.g2 is not None:
            g1 = acc.g1 if acc.g1.device == main.device else acc.g1.to(main.device)
            g2 = acc.g2 if acc.g2.device == main.device else acc.g2.to(main.device)
            inv = 1.0 / std
            if self._binary:
                # P holds r=1 sources, N holds r=0 sources
                if uniform:
                    axpby_(main, g1, g2, a_uni, a_uni)
                else:
                    axpby_(main, g1, g2, (1.0 - mean) * inv, -mean * inv)
            else:
                if uniform:
                    axpby_(main, g2, None, a_uni)
                else:
                    axpby_(main, g1, g2, inv, -mean * inv)
        n_b = max(len(acc.b2), len(acc.direct_boundary))
        for i in range(n_b):
            b1 = acc.b1[i] if i < len(acc.b1) else None
            b2 = acc.b2[i] if i < len(acc.b2) else None
            out = None
            if b2 is not None or b1 is not None:
                inv = 1.0 / std
                if self._binary:
                    p = b1 if b1 is not None else torch.zeros_like(b2)
                    n = b2 if b2 is not None else torch.zeros_like(b1)
                    if uniform:
                        out = (p + n) * a_uni
                    else:
                        out = p * ((1.0 - mean) * inv) + n * (-mean * inv)
                else:
                    if uniform:
                        out = b2 * a_uni
                    else:
                        bb1 = b1 if b1 is not None else torch.zeros_like(b2)
                        out = (bb1 - mean * b2) * inv
            d = acc.direct_boundary[i] if i < len(acc.direct_boundary) else None
            if d is not None:
                out = d if out is None else out + d
            adjoints.append(out)
        self._drop_stats(acc)
        acc.b1 = acc.b2 = []
        acc.direct_boundary = []
        boundary = self.run._groups[group_id].boundary
        if boundary is not None:
            full = adjoints + [None] * (len(boundary.real) - len(adjoints))
            self.run.finalize_group_boundary(group_id, full, sink=GradSink(self.arena, main))
        self.run.free_group(group_id)
        acc.done = True
        self._report["group_closes"] += 1

    # ------------------------------------------------------------ final work
    def close_final_forest(self, items: list[tuple[int, float]]) -> None:
        """Final trajectories (group fully bound): direct A_i·∇S_i backwards."""
        for tid, reward in items:
            self._record(int(tid), float(reward))
        for tid, reward in items:
            acc = self._acc(int(tid))
            if not self.group_fully_bound(acc.gid):
                raise RuntimeError(f"final work for trajectory {tid} needs its group fully bound")
            acc.direct = True
            self._differentiate(int(tid), float(reward), None)

    def cede_final_closes(self, traj_ids: list[int]) -> None:
        for tid in traj_ids:
            acc = self._acc(int(tid))
            acc.closed.add(int(tid))
            self.run.free_trajectory(int(tid))

    def backward_claimed_final(self, items: list[tuple[int, float]]) -> None:
        self.close_final_forest(items)

    # ------------------------------------------------------------ step gate
    def _check_versions(self) -> None:
        for p in self.run._trainable:
            if p._version != self._versions.get(id(p), p._version):
                raise RuntimeError(
                    "parameters changed inside a logical batch (version guard); step only after "
                    "assert_safe_to_step()"
                )

    def assert_safe_to_step(self, *, materialize: bool = True) -> None:
        """Refuse while any group is open; otherwise finish the batch gradient."""
        if self._aborted:
            raise RuntimeError("this backward was aborted")
        self._run_requested_closes(wait=True)
        open_ = [g for g, a in self._groups.items() if not a.done]
        if open_:
            raise RuntimeError(f"cannot step: groups {open_} are still open")
        self._check_versions()
        if self._host_fold is not None:
            self._host_fold.drain()
        main = self._main_grad()
        self.run.finalize_shared_prefixes(sink=GradSink(self.arena, main))
        self.run.materialize_parameter_adjoints()
        if materialize:
            self.materialize_grads()
        self._stepped = True

    def materialize_grads(self) -> None:
        """Write the flat fp32 batch gradient into ``param.grad`` (adding to any present)."""
        main = self._main
        if main is None:
            return
        with torch.no_grad():
            for p in self.run._trainable:
                v = self.arena.view(main, p)
                if p.grad is None:
                    p.grad = v.to(p.dtype, copy=True)
                else:
                    p.grad.add_(v.to(p.grad.dtype))

    def abort(self) -> None:
        self._aborted = True
        self._requested_closes = []
        if self._host_fold is not None:
            self._host_fold.drain()
            if self._host_fold_options.get("arena") is not None:
                self._host_fold.close()  # return the arena's slabs
            self._host_fold = None
        for gid, acc in self._groups.items():
            self._drop_stats(acc)
            acc.prepared.clear()
            self.run.free_group(gid)
            acc.done = True
        self._scratch = None

    # ------------------------------------------------------------ diagnostics
    def retained_device_bytes(self) -> dict[str, int]:
        stat = 0
        for a in self._groups.values():
            for t in (a.g1, a.g2):
                if t is not None and t.is_cuda:
                    stat += t.numel() * t.element_size()
        held = sum(s.numel() * s.element_size() for a in self._groups.values() for s, _ in a.prepared.values())
        main = 0 if self._main is None else self._main.numel() * 4
        scratch = 0 if self._scratch is None else self._scratch.numel() * 4
        return {"statistics": stat, "held_sources": held, "main_grad": main, "scratch": scratch,
                "total": stat + held + main + scratch}

    @property
    def source_offload_report(self) -> dict[str, Any]:
        out = {**self._report, **self._scope, "mode": self.source_offload_mode, "binary": self._binary}
        if self._host_fold is not None:
            out["host_fold"] = dict(self._host_fold.report)
        return out
