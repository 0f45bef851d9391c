"""DataParallelThunderSync: replicated, group-granular data-parallel GRPO (C37).

Each rank streams its own groups through a (StreamingRun, RewardLinearBackward)
pair; ranks communicate only at ``step()`` (reference:
src/thundersync/grpo/data_parallel.py:94-858). The global objective is the
mean over all N groups: each rank scales its local group sum (by 1/n_local
when counts are equal, by world/N otherwise) and the average all-reduce gives
the global mean.

B200-first differences:

* the batch gradient is the reward-linear objective's flat fp32 buffer in the
  parameter-arena layout, so the reduction is one contiguous range (reduced in
  buckets by :class:`thundersync_b200.parallel.reduce.GradientReducer`, which
  runs this package's NVLink kernels when peer memory is available and NCCL
  otherwise) and the count scale is folded into the reduction;
* with a :class:`~thundersync_b200.parallel.optimizer.FlatAdamW` the clip and
  the update run as fused flat kernels with no host synchronisation; a plain
  torch optimizer is also accepted (grads are materialised into
  ``param.grad`` first, the reference's behaviour);
* ``assert_safe_to_step`` runs locally before any collective, exactly as the
  reference requires, so a rank with open groups fails on its own.
"""

from __future__ import annotations

import contextlib
import datetime
import logging
import os
import time
from typing import Any, Callable, Iterator

import torch
import torch.distributed as dist

from thundersync_b200.engine.streaming import StreamingRun, arena_for
from thundersync_b200.grpo.config import DEFAULT_GRPO_EPSILON
from thundersync_b200.grpo.reward_linear import RewardLinearBackward
from thundersync_b200.parallel.optimizer import FlatAdamW, global_sq_norm

log = logging.getLogger(__name__)

__all__ = ["DataParallelThunderSync", "default_run_factory"]

RunFactory = Callable[[torch.nn.Module], StreamingRun]


def default_run_factory(model: torch.nn.Module) -> StreamingRun:
    """The production run: boundary cut, unstreamed turns, close-time rebuild."""
    return StreamingRun(model, boundary_cut=True, checkpoint=False, stream_turns=False)


def _init_process_group(device: torch.device, timeout_s: float) -> None:
    if dist.is_initialized():
        return
    backend = "nccl" if device.type == "cuda" else "gloo"
    kwargs: dict[str, Any] = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device.type == "cuda":
        kwargs["device_id"] = device
    dist.init_process_group(backend, **kwargs)


class DataParallelThunderSync:
    """One rank of the replicated data-parallel streaming GRPO trainer."""

    def __init__(
        self,
        model: torch.nn.Module,
        optimizer: Any,
        *,
        run_factory: RunFactory | None = None,
        eps: float = DEFAULT_GRPO_EPSILON,
        grad_clip: float | None = 1.0,
        source_offload_device: str | torch.device | None = "cpu",
        source_offload_mode: str = "blocking",
        source_offload_window_bytes: int = 256 * 1024 * 1024,
        source_offload_hbm_threshold: float = 0.65,
        source_reduction_mode: str = "unrestricted_statistics",
        source_reduction_pack_size: int = 1,
        source_reduction_worker_count: int = 2,
        source_offload_worker_count: int = 2,
        source_offload_pinned_windows: int = 2,
        source_spill_directory: Any = None,
        statistic_device: str | torch.device | None = None,
        device_statistic_slots: int | None = None,
        statistic_keep_source_dtype: bool = False,
        sharded_step: Any | None = None,
        retained_bytes_log_every: int = 0,
        source_pinned_arena: Any = None,
        direct_when_group_bound: bool = False,
        source_release_during_backward: bool = False,
        combine_known_reward_sources: bool = False,
        reducer: Any = None,
    ) -> None:
        if grad_clip is not None and grad_clip <= 0:
            raise ValueError("grad_clip must be positive when enabled")
        self.model = model
        self.optimizer = optimizer
        self._sharded_step = sharded_step
        self.run_factory = run_factory or default_run_factory
        self.eps = eps
        self.grad_clip = grad_clip
        self._bw_kwargs = dict(
            eps=eps,
            source_offload_device=source_offload_device,
            source_offload_mode=source_offload_mode,
            source_offload_window_bytes=source_offload_window_bytes,
            source_offload_hbm_threshold=source_offload_hbm_threshold,
            source_reduction_mode=source_reduction_mode,
            source_reduction_pack_size=source_reduction_pack_size,
            source_reduction_worker_count=source_reduction_worker_count,
            source_offload_worker_count=source_offload_worker_count,
            source_offload_pinned_windows=source_offload_pinned_windows,
            source_spill_directory=source_spill_directory,
            statistic_device=statistic_device,
            device_statistic_slots=device_statistic_slots,
            statistic_keep_source_dtype=statistic_keep_source_dtype,
            source_pinned_arena=source_pinned_arena,
            direct_when_group_bound=direct_when_group_bound,
            source_copy_during_backward=source_release_during_backward,
            source_release_during_backward=source_release_during_backward,
            combine_known_reward_sources=combine_known_reward_sources,
        )
        self.source_pinned_arena = source_pinned_arena
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.world_size = dist.get_world_size() if dist.is_initialized() else 1
        self.device = next(model.parameters()).device
        self._trainable = [p for p in model.parameters() if p.requires_grad]
        self.arena = arena_for(model)
        if self.arena is None:
            raise ValueError("trainable parameters must share one device and dtype")
        self._sharded_flat = isinstance(optimizer, FlatAdamW) and optimizer.is_sharded
        if reducer is None and self.world_size > 1:
            from thundersync_b200.parallel.reduce import GradientReducer

            reducer = GradientReducer(self.arena.numel, self.device, arena=self.arena,
                                      shard_params=self._sharded_flat)
        self.reducer = reducer
        self._binary_rewards = False
        self._steps_done = 0
        self._shutdown = False
        self._retained_bytes_log_every = int(retained_bytes_log_every)
        self._retained_events = 0
        self._final_forest: tuple[int, int] | None = None
        self._price_attention_weight: float | None = None
        self._work_claims_report: dict[str, Any] | None = None
        # True: step() synchronises the device around its phases so allreduce_s / opt_step_s are device
        # times; False (default): they are host issue times and the step adds no synchronisation
        self.step_timing = False
        self._new_batch()

    # ------------------------------------------------------------ construction
    @classmethod
    def init_from_env(
        cls,
        model: torch.nn.Module,
        optimizer: Any,
        *,
        timeout_s: float = 600.0,
        **kwargs: Any,
    ) -> "DataParallelThunderSync":
        """Join (or create) the process group from torchrun's env and broadcast rank 0's weights."""
        device = next(model.parameters()).device
        if device.type == "cuda":
            torch.cuda.set_device(device)
        if "WORLD_SIZE" in os.environ or dist.is_initialized():
            _init_process_group(device, timeout_s)
        if dist.is_initialized() and dist.get_world_size() > 1:
            arena = arena_for(model)
            with torch.no_grad():
                if arena is not None:
                    dist.broadcast(arena.flat, src=0)
                seen = set() if arena is None else set(arena.offsets)
                for t in list(model.state_dict(keep_vars=True).values()):
                    if id(t) in seen or not isinstance(t, torch.Tensor):
                        continue
                    dist.broadcast(t.data, src=0)
            if isinstance(optimizer, FlatAdamW):
                optimizer.master.copy_(optimizer.arena.flat[optimizer.lo : optimizer.hi].float())
        return cls(model, optimizer, **kwargs)

    # ------------------------------------------------------------ failure handling
    @contextlib.contextmanager
    def _abort_on_failure(self) -> Iterator[None]:
        try:
            yield
        except BaseException as exc:
            # the event's own error is the one to see; an abort that also fails is noted on it
            try:
                self.bw.abort()
            except BaseException as abort_exc:  # noqa: BLE001
                exc.add_note(f"aborting the backward after this error also failed: {abort_exc!r}")
            raise

    # ------------------------------------------------------------ events
    def open_group(self, group_id: int, prompt_tokens: list[int]) -> None:
        with self._abort_on_failure():
            self.run.open_group(group_id, prompt_tokens)

    def open_groups_shared_prefix(self, groups) -> None:
        with self._abort_on_failure():
            self.run.open_groups_shared_prefix(groups)

    def register_group_trajectories(self, group_id: int, trajectory_ids: list[int]) -> None:
        self.bw.register_group_trajectories(group_id, trajectory_ids)

    def append_turn(self, group_id: int, traj_id: int, tokens: list[int], scored: list[bool]) -> None:
        with self._abort_on_failure():
            self.run.append_turn(group_id, traj_id, tokens, scored)

    def append_turns(self, items, *, joint_backward: bool = False) -> None:
        with self._abort_on_failure():
            self.run.append_turns(items, joint_backward=joint_backward)

    def close_trajectory(self, traj_id: int, reward: float, token_weights=None) -> None:
        with self._abort_on_failure():
            self.bw.close_trajectory(traj_id, reward, token_weights)
        self._sample_retained("close_trajectory")

    def close_trajectories(self, items) -> None:
        for item in items:
            if item[1] is None:
                raise ValueError(f"trajectory {item[0]} closed without a reward")
        with self._abort_on_failure():
            self.bw.close_trajectories(items)

    def prepare_trajectories(self, trajectory_ids) -> None:
        with self._abort_on_failure():
            self.bw.prepare_trajectories(trajectory_ids)

    def bind_rewards(self, items) -> None:
        for tid, reward in items:
            if reward is None:
                raise ValueError(
                    f"trajectory {tid} bound without a reward; a missing coefficient is a wiring error"
                )
        with self._abort_on_failure():
            self.bw.bind_rewards(items)

    def record_rewards(self, items) -> None:
        for tid, reward in items:
            if reward is None:
                raise ValueError(f"trajectory {tid} recorded without a reward")
        self.bw.record_rewards(items)

    def group_fully_bound(self, group_id: int) -> bool:
        return self.bw.group_fully_bound(group_id)

    def registered_groups_fully_bound(self) -> bool:
        return self.bw.registered_groups_fully_bound()

    def group_reduction_complete(self, group_id: int) -> bool:
        return self.bw.group_reduction_complete(group_id)

    def wait_for_trajectory_reduction(self, group_id: int, trajectory_id: int) -> None:
        self.bw.wait_for_trajectory_reduction(group_id, trajectory_id)

    def close_group(self, group_id: int) -> None:
        with self._abort_on_failure():
            self.bw.close_group(group_id)
        self._local_groups_closed += 1

    def configure_binary_rewards(self) -> None:
        self._binary_rewards = True
        self.bw.configure_binary_rewards()

    def set_statistics_branch_observer(self, observer) -> None:
        self.bw.set_statistics_branch_observer(observer)

    # ------------------------------------------------------------ final work
    def configure_final_forest(self, max_tokens_per_microbatch: int, chunk: int = 1024) -> None:
        """Token cap of the final forest's micro-batches (claimed peer work) and of a claim chunk; ``chunk``
        is the LM head's rows per block in those forwards."""
        if max_tokens_per_microbatch <= 0 or chunk <= 0:
            raise ValueError("the final forest's token cap and chunk must be positive")
        if not self.bw.direct_when_group_bound:
            raise ValueError("the final forest runs direct closes: construct with direct_when_group_bound=True")
        self._final_forest = (int(max_tokens_per_microbatch), int(chunk))

    @property
    def final_forest_max_tokens(self) -> int:
        if self._final_forest is None:
            raise RuntimeError("the final forest is not configured")
        return self._final_forest[0]

    @property
    def final_forest_enabled(self) -> bool:
        return self._final_forest is not None

    def close_final_forest(self, items) -> None:
        with self._abort_on_failure():
            self.bw.close_final_forest(items)

    def cede_final_closes(self, items) -> None:
        self.bw.cede_final_closes([t for t, _ in items])

    def final_work(self, trajectory_id: int) -> tuple[int, int, bytes]:
        from thundersync_b200.grpo.claims import encode_final_work
        from thundersync_b200.grpo.work_price import attention_weight, trajectory_price

        gid = self.bw._traj_group[trajectory_id]
        prompt = self.run._groups[gid].prompt
        t = self.run._trajs[trajectory_id]
        adv = self.bw.final_advantage(trajectory_id)
        payload = encode_final_work(group_id=gid, trajectory_id=trajectory_id, advantage=adv,
                                    prompt_tokens=prompt, turns=t.turns)
        if self._price_attention_weight is None:
            n = sum(p.numel() for p in self.model.parameters())
            self._price_attention_weight = attention_weight(self.model.config, n)
        turn_tokens = sum(len(tk) for tk, _ in t.turns)
        price = trajectory_price(len(prompt), turn_tokens, self._price_attention_weight)
        return len(prompt) + turn_tokens, int(price), payload

    def run_claimed_work(self, payloads: list[bytes]) -> None:
        from thundersync_b200.grpo.final_forest import backward_claimed_payloads

        with self._abort_on_failure():
            backward_claimed_payloads(self, payloads)

    def record_work_claims(self, report: dict[str, Any]) -> None:
        self._work_claims_report = dict(report)

    @property
    def local_groups_closed(self) -> int:
        return self._local_groups_closed

    @property
    def optimizer_steps_completed(self) -> int:
        return self._steps_done

    # ------------------------------------------------------------ step
    def step(self, *, gradient_observer: Callable | None = None) -> dict:
        """The one collective point: average the batch gradient across ranks, then update.

        1. ``assert_safe_to_step`` locally (no collective yet);
        2. group counts: one small all-reduce;
        3. scale folded into the reduction: 1/n_local (equal counts) or world/N;
        4. flat fp32 gradient averaged across ranks (bucketed);
        5. global-norm clip coefficient on the device, fused AdamW update
           (or a torch optimizer on materialised grads);
        6. fresh run and objective for the next batch.
        """
        self.bw.assert_safe_to_step(materialize=False)
        stats: dict[str, Any] = {"rank": self.rank, "world_size": self.world_size,
                                 "n_local_groups": self._local_groups_closed}
        # device-synchronised phase timings only on request (each synchronisation drains the queue)
        sync = self.device.type == "cuda" and self.step_timing
        if sync:
            torch.cuda.synchronize(self.device)
        t0 = time.perf_counter()
        counts = torch.zeros(self.world_size, dtype=torch.long, device=self.device)
        counts[self.rank] = self._local_groups_closed
        if self.world_size > 1:
            dist.all_reduce(counts, op=dist.ReduceOp.SUM)
        counts_l = counts.tolist()
        n_local = counts_l[self.rank]
        n_global = sum(counts_l)
        if n_global < 1 or any(c < 1 for c in counts_l):
            raise RuntimeError(f"invalid groups across ranks: {counts_l}")
        scale = 1.0 / n_local if len(set(counts_l)) == 1 else self.world_size / n_global
        grad = self.bw.main_grad()
        if grad is None:
            grad = self.arena.new_buffer(torch.float32)
        if self._sharded_step is not None:
            # a caller-built ShardedOptimizerStep (engine/sharded_step.py) owns reduction, clipping and the
            # step over replicated p.grad (reference src/thundersync/grpo/data_parallel.py:721-735)
            if gradient_observer is not None:
                raise RuntimeError("gradient observers are not supported under the sharded optimizer step")
            with torch.no_grad():
                for p in self._trainable:
                    p.grad = (self.arena.view(grad, p) * scale).to(p.dtype)
            shard_stats = self._sharded_step.step()
            t2 = time.perf_counter()
            stats["n_global_groups"] = n_global
            stats["group_counts_by_rank"] = counts_l
            stats["local_gradient_scale"] = scale
            stats["grad_bytes"] = grad.numel() * grad.element_size()
            for k in ("allreduce_s", "global_grad_norm", "grad_clip", "gradient_was_clipped", "opt_step_s"):
                stats[k] = shard_stats[k]
            stats["sharded_step"] = shard_stats
        else:
            t2 = self._replicated_or_flat_step(grad, scale, stats, n_global, counts_l, gradient_observer, sync)
        if self.reducer is not None:
            self.reducer.check()
        if sync:
            torch.cuda.synchronize(self.device)
        t3 = time.perf_counter()
        if self._sharded_step is None:
            stats["opt_step_s"] = t3 - t2
        stats["step_total_s"] = t3 - t0
        stats["source_offload_report"] = self.bw.source_offload_report
        stats["rebuild_path_counts"] = self.run.rebuild_path_counts
        if self._work_claims_report is not None:
            stats["work_claims"] = self._work_claims_report
        stats["run_retained_bytes"] = self.run.retained_device_bytes()
        stats["backward_retained_bytes"] = self.bw.retained_device_bytes()
        if sync:
            a = torch.cuda.memory_stats(self.device)
            stats["cuda_allocator"] = {k: a.get(k) for k in ("num_alloc_retries", "num_ooms", "num_device_alloc",
                                                              "num_device_free", "num_sync_all_streams")}
        self._steps_done += 1
        self._new_batch()
        return stats

    def _replicated_or_flat_step(self, grad, scale, stats, n_global, counts_l, gradient_observer, sync) -> float:
        """Reduce the flat gradient (or reduce-scatter it under the sharded flat AdamW), clip, step; returns
        the time the reduction ended."""
        t1 = time.perf_counter()
        norm_t = None
        if self._sharded_flat:
            norm_t = self._sharded_update(grad, scale)
        else:
            if self.world_size > 1:
                self.reducer.all_reduce_mean(grad, pre_scale=scale)
            else:
                from thundersync_b200.ops.fold import scale_

                scale_(grad, scale) if grad.is_cuda else grad.mul_(scale)
        if sync:
            torch.cuda.synchronize(self.device)
        t2 = time.perf_counter()
        stats["allreduce_s"] = t2 - t1
        stats["n_global_groups"] = n_global
        stats["group_counts_by_rank"] = counts_l
        stats["local_gradient_scale"] = scale
        stats["grad_bytes"] = grad.numel() * grad.element_size()
        stats["reduction_path"] = None if self.reducer is None else self.reducer.last_path
        if gradient_observer is not None:
            gradient_observer("raw_reduced", grad)
        if norm_t is not None:
            norm_value = float(norm_t)
        elif isinstance(self.optimizer, FlatAdamW):
            sq = global_sq_norm(grad)
            coef, nrm = self.optimizer.clip_coefficient(sq, self.grad_clip)
            self.optimizer.step(grad, clip_coef=coef)
            norm_value = float(nrm)
        else:
            with torch.no_grad():
                for p in self._trainable:
                    p.grad = self.arena.view(grad, p).to(p.dtype, copy=True)
            nrm = torch.nn.utils.clip_grad_norm_(
                self._trainable, self.grad_clip if self.grad_clip is not None else float("inf"), foreach=False
            )
            norm_value = float(nrm)
            self.optimizer.step()
            self.optimizer.zero_grad(set_to_none=True)
        stats["global_grad_norm"] = norm_value
        stats["grad_clip"] = self.grad_clip
        stats["gradient_was_clipped"] = self.grad_clip is not None and norm_value > self.grad_clip
        return t2

    def _sharded_update(self, grad: torch.Tensor, scale: float):
        """ZeRO-1: reduce-scatter, shard-local AdamW, parameter all-gather."""
        opt: FlatAdamW = self.optimizer
        red = self.reducer
        if red is not None and red.native and red.main_grad_buffer() is not None \
                and grad.data_ptr() == red.main_grad_buffer().data_ptr():
            lo, hi = red.reduce_scatter_mean(grad, pre_scale=scale)
            if (lo, hi) != (opt.lo, opt.hi):
                raise RuntimeError("optimizer shard differs from the reduction shard")
            norm = opt.step_gather(grad[lo:hi], red.param_ptrs, red.ws.norm_slots, self.grad_clip)
            red.ws.barrier(2)
            return norm
        # portable path: all-reduce, local clip, shard update, parameter all-gather
        if red is not None:
            red.all_reduce_mean(grad, pre_scale=scale)
        sq = global_sq_norm(grad)
        coef, nrm = opt.clip_coefficient(sq, self.grad_clip)
        opt.step(grad[opt.lo:opt.hi], clip_coef=coef)
        if self.world_size > 1:
            from thundersync_b200.parallel.symm import shard_bounds

            chunk = shard_bounds(self.arena.numel, self.world_size, 0)[1]
            buf = torch.zeros(chunk * self.world_size, dtype=self.arena.dtype, device=self.arena.device)
            mine = buf[self.rank * chunk : self.rank * chunk + (opt.hi - opt.lo)]
            mine.copy_(self.arena.flat[opt.lo:opt.hi])
            dist.all_gather_into_tensor(buf, buf[self.rank * chunk : (self.rank + 1) * chunk].clone())
            with torch.no_grad():
                self.arena.flat.copy_(buf[: self.arena.numel])
        return nrm

    def shutdown(self) -> None:
        if self._shutdown:
            return
        try:
            self.bw.abort()
        finally:
            if self.reducer is not None and hasattr(self.reducer, "close"):
                self.reducer.close()
            self._shutdown = True

    # ------------------------------------------------------------ internal
    def _new_batch(self) -> None:
        old = getattr(self, "run", None)
        if old is not None:
            old.close()
        self.run = self.run_factory(self.model)
        self.bw = RewardLinearBackward(self.run, self.model, **self._bw_kwargs)
        buf = None if self.reducer is None else self.reducer.main_grad_buffer()
        if buf is not None:
            self.bw.use_main_grad_buffer(buf)
        if self._binary_rewards:
            self.bw.configure_binary_rewards()
        self.bw.set_diagnostic_scope(rank=self.rank, step=self._steps_done + 1)
        self._local_groups_closed = 0
        self._work_claims_report = None

    def retained_device_bytes(self) -> dict[str, Any]:
        return {"run": self.run.retained_device_bytes(), "backward": self.bw.retained_device_bytes()}

    def _sample_retained(self, event: str) -> None:
        if self._retained_bytes_log_every <= 0:
            return
        self._retained_events += 1
        if self._retained_events % self._retained_bytes_log_every == 0:
            log.info("retained %s %s", event, self.retained_device_bytes())
