"""ZeRO-1 optimizer-state sharding behind an injectable collectives seam (C39).

Parameters and gradients stay replicated; each rank builds its optimizer over
a contiguous, numel-balanced shard of the canonical trainable-parameter order
and steps only that shard (reference: src/thundersync/engine/sharded_step.py:
1-559). ``step()``:

1. average the gradients across ranks (one flat collective per dtype);
2. clip over *all* parameters — replicated gradients make the local norm the
   global norm — and check with one all-gather that every rank computed the
   bitwise-same norm (fails closed on replica drift);
3. ``optimizer.step()`` on the owned shard (AdamW is a per-parameter map, so
   the shard update equals the matching slice of an unsharded step);
4. re-synchronise the replicas by broadcasting each owner's updated shard
   (one flat broadcast per owner).

The partition is a pure function of (parameter numels, world size), so every
rank derives the same one from the same canonical order; a SHA-256 digest of
(shard, name, shape, dtype) is all-gathered at construction and any mismatch
raises. ``world_size == 1`` runs no collective at all.

This is the generic, any-optimizer path. The data-parallel GRPO trainer's
fast path shards a flat parameter arena instead and runs its reduce-scatter,
fused AdamW and parameter all-gather as this package's peer-memory kernels
(:mod:`thundersync_b200.parallel`).
"""

from __future__ import annotations

import bisect
import hashlib
import time
from typing import Callable, Sequence

import torch
import torch.distributed as dist
from torch._utils import _flatten_dense_tensors, _unflatten_dense_tensors

__all__ = ["Collectives", "OptimizerFactory", "ShardedOptimizerStep", "TorchDistributedCollectives",
           "partition_contiguous_by_numel"]

OptimizerFactory = Callable[[list[torch.nn.Parameter]], torch.optim.Optimizer]
_MISSING = ("error", "zero")


def partition_contiguous_by_numel(numels: Sequence[int], world_size: int) -> tuple[tuple[int, int], ...]:
    """``world_size`` contiguous, non-empty, numel-balanced spans of ``range(len(numels))``.

    Boundary ``s`` sits at the prefix-sum point nearest ``s/world_size`` of
    the total (the smaller index on a tie), constrained so that every shard
    keeps at least one parameter.
    """
    if world_size < 1:
        raise ValueError(f"world_size must be >= 1, got {world_size}")
    if any(n <= 0 for n in numels):
        raise ValueError("every parameter must have positive numel")
    count = len(numels)
    if count < world_size:
        raise ValueError(f"cannot partition {count} parameters into {world_size} non-empty shards")
    if world_size == 1:
        return ((0, count),)
    prefix = [0]
    for n in numels:
        prefix.append(prefix[-1] + n)
    total = prefix[-1]
    cuts = [0]
    for s in range(1, world_size):
        target = total * s / world_size
        lo, hi = cuts[-1] + 1, count - (world_size - s)
        j = bisect.bisect_left(prefix, target, lo, hi + 1)  # first cut whose prefix >= target
        best = min(max(j, lo), hi)
        if best > lo and abs(prefix[best - 1] - target) <= abs(prefix[best] - target):
            best -= 1
        cuts.append(best)
    cuts.append(count)
    return tuple((cuts[i], cuts[i + 1]) for i in range(world_size))


def _digest(names: Sequence[str], params: Sequence[torch.Tensor], spans) -> int:
    h = hashlib.sha256()
    for shard, (a, b) in enumerate(spans):
        for i in range(a, b):
            h.update(f"{shard}\t{names[i]}\t{tuple(params[i].shape)}\t{params[i].dtype}\n".encode())
    return int.from_bytes(h.digest()[:8], "big", signed=True)


class Collectives:
    """In-place collectives; identical results and call sequences on every rank."""

    def all_reduce_average_(self, tensor: torch.Tensor) -> None:
        raise NotImplementedError

    def broadcast_(self, tensor: torch.Tensor, source_rank: int) -> None:
        raise NotImplementedError

    def all_gather_(self, outputs: list[torch.Tensor], tensor: torch.Tensor) -> None:
        raise NotImplementedError

    def all_reduce_averages_(self, tensors: Sequence[torch.Tensor]) -> None:
        for t in tensors:
            self.all_reduce_average_(t)

    def broadcasts_(self, tensors: Sequence[torch.Tensor], source_ranks: Sequence[int]) -> None:
        for t, r in zip(tensors, source_ranks, strict=True):
            self.broadcast_(t, r)


class TorchDistributedCollectives(Collectives):
    """``torch.distributed`` backend: one flat bucket per dtype / per owner instead of one call per tensor."""

    def __init__(self, process_group: object | None = None) -> None:
        if not dist.is_initialized():
            raise RuntimeError("TorchDistributedCollectives requires an initialized process group; initialize "
                               "torch.distributed before constructing a sharded step, or inject a Collectives backend")
        self._group = process_group
        self._world = dist.get_world_size(process_group)

    def all_reduce_average_(self, tensor: torch.Tensor) -> None:
        dist.all_reduce(tensor, op=dist.ReduceOp.SUM, group=self._group)
        tensor.div_(self._world)

    def broadcast_(self, tensor: torch.Tensor, source_rank: int) -> None:
        dist.broadcast(tensor, src=source_rank, group=self._group)

    def all_gather_(self, outputs: list[torch.Tensor], tensor: torch.Tensor) -> None:
        dist.all_gather(outputs, tensor, group=self._group)

    def all_reduce_averages_(self, tensors: Sequence[torch.Tensor]) -> None:
        by_dtype: dict[torch.dtype, list[torch.Tensor]] = {}
        for t in tensors:
            by_dtype.setdefault(t.dtype, []).append(t)
        for dt in sorted(by_dtype, key=str):  # same order on every rank
            group = by_dtype[dt]
            flat = _flatten_dense_tensors(group)
            self.all_reduce_average_(flat)
            for t, v in zip(group, _unflatten_dense_tensors(flat, group)):
                t.copy_(v)

    def broadcasts_(self, tensors: Sequence[torch.Tensor], source_ranks: Sequence[int]) -> None:
        owners: dict[tuple[int, torch.dtype], list[torch.Tensor]] = {}
        for t, r in zip(tensors, source_ranks, strict=True):
            owners.setdefault((r, t.dtype), []).append(t)
        for key in sorted(owners, key=lambda k: (k[0], str(k[1]))):
            group = owners[key]
            flat = _flatten_dense_tensors(group)
            self.broadcast_(flat, key[0])
            for t, v in zip(group, _unflatten_dense_tensors(flat, group)):
                t.copy_(v)


class ShardedOptimizerStep:
    """Replicated parameters and gradients, optimizer state for this rank's shard only."""

    def __init__(self, named_parameters: Sequence[tuple[str, torch.nn.Parameter]], optimizer_factory: OptimizerFactory,
                 *, world_size: int, rank: int, collectives: Collectives | None = None,
                 grad_clip: float | None = None, missing_grad_policy: str = "error") -> None:
        if world_size < 1:
            raise ValueError(f"world_size must be >= 1, got {world_size}")
        if not 0 <= rank < world_size:
            raise ValueError(f"rank {rank} outside [0, {world_size})")
        if grad_clip is not None and grad_clip <= 0:
            raise ValueError("grad_clip must be positive when enabled")
        if missing_grad_policy not in _MISSING:
            raise ValueError(f"missing_grad_policy must be one of {_MISSING}, got {missing_grad_policy!r}")
        pairs = list(named_parameters)
        if not pairs:
            raise ValueError("named_parameters is empty")
        names = [n for n, _ in pairs]
        params = [p for _, p in pairs]
        if len(set(names)) != len(names):
            raise ValueError("duplicate parameter names in canonical order")
        if len({id(p) for p in params}) != len(params):
            raise ValueError("aliased parameter objects in canonical order; tied weights must appear exactly once")
        for n, p in pairs:
            if not p.requires_grad:
                raise ValueError(f"parameter {n!r} has requires_grad=False; pass only trainable parameters")
        devices = {p.device for p in params}
        if len(devices) != 1:
            raise ValueError(f"parameters span multiple devices {sorted(map(str, devices))}")
        self._names, self._params = tuple(names), params
        self._world, self._rank = world_size, rank
        self._clip = grad_clip
        self._missing = missing_grad_policy
        self._device = params[0].device
        self._steps = 0
        self._spans = partition_contiguous_by_numel([p.numel() for p in params], world_size)
        a, b = self._spans[rank]
        self._owned = params[a:b]
        self._owned_names = tuple(names[a:b])
        self._owner = [s for s, (x, y) in enumerate(self._spans) for _ in range(x, y)]
        self._optimizer = optimizer_factory(list(self._owned))
        captured = {id(p) for g in self._optimizer.param_groups for p in g["params"]}
        owned = {id(p) for p in self._owned}
        if captured != owned:
            raise ValueError("optimizer_factory must build an optimizer over exactly the owned shard; it captured "
                             f"{len(captured - owned)} foreign and missed {len(owned - captured)} owned parameters")
        self._coll: Collectives | None = None
        if world_size > 1:
            self._coll = collectives if collectives is not None else TorchDistributedCollectives()
            self._check_partition()

    # ---------------------------------------------------------------- inspection
    @property
    def optimizer(self) -> torch.optim.Optimizer:
        return self._optimizer

    @property
    def partition_spans(self) -> tuple[tuple[int, int], ...]:
        return self._spans

    @property
    def owned_parameters(self) -> tuple[torch.nn.Parameter, ...]:
        return tuple(self._owned)

    @property
    def owned_parameter_names(self) -> tuple[str, ...]:
        return self._owned_names

    @property
    def optimizer_steps_completed(self) -> int:
        return self._steps

    def retained_device_bytes(self) -> dict[str, int]:
        """Device bytes held: replicated parameters and the owned shard's optimizer state."""
        def nbytes(ts):
            return sum(t.numel() * t.element_size() for t in ts if t.device == self._device)

        state = [v for s in self._optimizer.state.values() for v in s.values() if torch.is_tensor(v)]
        return {"_parameters": nbytes(self._params), "_optimizer": nbytes(state)}

    # ---------------------------------------------------------------------- step
    def _sync(self) -> None:
        if self._device.type == "cuda":
            torch.cuda.synchronize(self._device)

    def _need(self) -> Collectives:
        if self._coll is None:
            raise RuntimeError(f"world_size={self._world} step has no collectives")
        return self._coll

    def _check_partition(self) -> None:
        d = _digest(self._names, self._params, self._spans)
        local = torch.tensor([d], dtype=torch.int64, device=self._device)
        got = [torch.zeros_like(local) for _ in range(self._world)]
        self._need().all_gather_(got, local)
        vals = [int(t.item()) for t in got]
        if any(v != d for v in vals):
            raise RuntimeError(f"partition drift across ranks: rank {self._rank} digest {d} vs gathered {vals}; every "
                               "rank must construct ShardedOptimizerStep from the identical canonical parameter order")

    def _check_norm(self, norm: torch.Tensor) -> None:
        if not bool(torch.isfinite(norm)):
            raise RuntimeError(f"non-finite global grad norm {float(norm)}; refusing the sharded step")
        local = norm.detach().reshape(1).clone()
        got = [torch.zeros_like(local) for _ in range(self._world)]
        self._need().all_gather_(got, local)
        for r, other in enumerate(got):
            if not torch.equal(other, local):
                raise RuntimeError(f"global grad norm disagrees across ranks: rank {self._rank} computed "
                                   f"{float(local)} but rank {r} computed {float(other)}; replicas have diverged")

    def _preconditions(self) -> None:
        missing = []
        for n, p in zip(self._names, self._params, strict=True):
            if not p.requires_grad:
                raise RuntimeError(f"parameter {n!r} lost requires_grad after construction; the partition and "
                                   "optimizer shard are frozen at construction time")
            if p.grad is None:
                missing.append(n)
        if not missing:
            return
        if self._missing == "error":
            raise RuntimeError(f"{len(missing)} parameters have no gradient (first: {missing[0]!r}); pass "
                               "missing_grad_policy='zero' only if a zero contribution is the declared semantics")
        with torch.no_grad():
            for p in self._params:
                if p.grad is None:
                    p.grad = torch.zeros_like(p)

    def step(self) -> dict[str, object]:
        self._preconditions()
        self._sync()
        t0 = time.perf_counter()
        if self._world > 1:
            self._need().all_reduce_averages_([p.grad for p in self._params])
        self._sync()
        t1 = time.perf_counter()
        norm = torch.nn.utils.clip_grad_norm_(self._params, self._clip if self._clip is not None else float("inf"),
                                              foreach=False)
        if self._world > 1:
            self._check_norm(norm)
        self._sync()
        t2 = time.perf_counter()
        self._optimizer.step()
        self._sync()
        t3 = time.perf_counter()
        moved = 0
        if self._world > 1:
            with torch.no_grad():
                self._need().broadcasts_([p.data for p in self._params], self._owner)
            moved = sum(p.numel() * p.element_size() for p in self._params)
        for p in self._params:
            p.grad = None
        self._sync()
        t4 = time.perf_counter()
        gn = float(norm.detach())
        self._steps += 1
        return {
            "rank": self._rank, "world_size": self._world, "n_params": len(self._params),
            "global_grad_norm": gn, "grad_clip": self._clip,
            "gradient_was_clipped": self._clip is not None and gn > self._clip,
            "owned_param_count": len(self._owned), "owned_param_numel": sum(p.numel() for p in self._owned),
            "owned_param_bytes": sum(p.numel() * p.element_size() for p in self._owned),
            "broadcast_bytes": moved, "allreduce_collectives": len(self._params) if self._world > 1 else 0,
            "allreduce_s": t1 - t0, "clip_s": t2 - t1, "opt_step_s": t3 - t2, "broadcast_s": t4 - t3,
            "step_total_s": t4 - t0,
        }
