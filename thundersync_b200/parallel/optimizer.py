"""Flat AdamW over the parameter arena: fp32 master, fp32 moments, fused clip.

One fused kernel updates a contiguous range of the arena: it scales the fp32
gradient by the global-norm clip coefficient (computed on the device, no host
sync), applies AdamW (decoupled weight decay, bias correction, optional
``maximize`` for GRPO) to the fp32 master and writes the rounded model copy
in place. With ``shard=(lo, hi)`` only that range's master and moments exist
on this rank (the ZeRO-1 partition); the caller all-gathers parameters.

Update rule and defaults follow ``torch.optim.AdamW`` (the reference builds
``AdamW(lr, betas=(0.9, 0.999), eps=1e-8, weight_decay=0, maximize=True)``,
src/thundersync/grpo/runtime.py:220-228).
"""

from __future__ import annotations

import torch

from thundersync_b200.ops._ext import native
from thundersync_b200.ops.sink import ParamArena

__all__ = ["FlatAdamW", "global_sq_norm"]


def global_sq_norm(grad: torch.Tensor) -> torch.Tensor:
    """Squared L2 norm of an fp32 flat buffer as a 1-element device tensor."""
    if grad.is_cuda:
        return native().sq_norm(grad)
    return grad.double().pow(2).sum().float().reshape(1)


class FlatAdamW:
    def __init__(
        self,
        arena: ParamArena,
        *,
        lr: float,
        betas: tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 0.0,
        maximize: bool = False,
        shard: tuple[int, int] | None = None,
    ) -> None:
        if lr <= 0:
            raise ValueError("lr must be positive")
        self.arena = arena
        self.lr = float(lr)
        self.betas = (float(betas[0]), float(betas[1]))
        self.eps = float(eps)
        self.weight_decay = float(weight_decay)
        self.maximize = bool(maximize)
        lo, hi = shard if shard is not None else (0, arena.numel)
        if not 0 <= lo <= hi <= arena.numel:
            raise ValueError("shard range outside the arena")
        self.lo, self.hi = lo, hi
        self.master = arena.flat[lo:hi].detach().float().clone()
        self.exp_avg = torch.zeros_like(self.master)
        self.exp_avg_sq = torch.zeros_like(self.master)
        self.steps = 0
        self.last_norm: torch.Tensor | None = None

    @classmethod
    def sharded(cls, arena: ParamArena, **kw) -> "FlatAdamW":
        """ZeRO-1: own only this rank's contiguous shard of the arena (requires a process group)."""
        import torch.distributed as dist

        from thundersync_b200.parallel.symm import shard_bounds

        world = dist.get_world_size() if dist.is_initialized() else 1
        rank = dist.get_rank() if dist.is_initialized() else 0
        return cls(arena, shard=shard_bounds(arena.numel, world, rank), **kw)

    @property
    def is_sharded(self) -> bool:
        return (self.lo, self.hi) != (0, self.arena.numel)

    def step_gather(self, grad_shard: torch.Tensor, param_ptrs: list[int], norm_slots: torch.Tensor,
                    max_norm: float | None) -> torch.Tensor:
        """Fused AdamW on this shard that writes bf16 params into every rank's arena (native path).

        ``norm_slots`` holds each rank's squared shard norm; the clip
        coefficient is formed on the device. Returns the global norm (device).
        """
        self.steps += 1
        b1, b2 = self.betas
        norm = torch.empty(1, dtype=torch.float32, device=self.master.device)
        native().symm_adamw_gather(
            self.master, self.exp_avg, self.exp_avg_sq, grad_shard, param_ptrs, self.lo, self.lr, b1, b2,
            self.eps, self.weight_decay, self.steps, self.maximize, norm_slots,
            -1.0 if max_norm is None else float(max_norm), norm,
        )
        with torch.no_grad():
            self.arena.flat[:0].add_(0)
        return norm

    @property
    def param_groups(self):  # enough of torch's optimizer surface for schedulers/loggers
        return [{"lr": self.lr, "betas": self.betas, "eps": self.eps, "weight_decay": self.weight_decay,
                 "maximize": self.maximize}]

    def state_dict(self) -> dict:
        return {"lo": self.lo, "hi": self.hi, "steps": self.steps, "master": self.master,
                "exp_avg": self.exp_avg, "exp_avg_sq": self.exp_avg_sq, "lr": self.lr,
                "betas": self.betas, "eps": self.eps, "weight_decay": self.weight_decay,
                "maximize": self.maximize}

    def load_state_dict(self, sd: dict) -> None:
        if (sd["lo"], sd["hi"]) != (self.lo, self.hi):
            raise ValueError("optimizer shard range differs from the checkpoint's")
        self.master.copy_(sd["master"])
        self.exp_avg.copy_(sd["exp_avg"])
        self.exp_avg_sq.copy_(sd["exp_avg_sq"])
        self.steps = int(sd["steps"])
        with torch.no_grad():
            self.arena.flat[self.lo : self.hi].copy_(self.master.to(self.arena.dtype))

    def step(self, grad: torch.Tensor, *, clip_coef: torch.Tensor | None = None) -> None:
        """Apply one update with ``grad`` (fp32, this shard's range, arena layout).

        ``clip_coef`` is a 1-element device tensor multiplied into the gradient.
        """
        if grad.numel() != self.hi - self.lo:
            raise ValueError("gradient does not cover this optimizer's range")
        self.steps += 1
        b1, b2 = self.betas
        param = self.arena.flat[self.lo : self.hi]
        if param.is_cuda:
            native().adamw_flat(
                self.master, param, grad, self.exp_avg, self.exp_avg_sq, self.lr, b1, b2, self.eps,
                self.weight_decay, self.steps, clip_coef, 1.0, self.maximize,
            )
            # kernel writes bypass autograd's version counter; bump it so saved
            # views from before the step are recognised as stale
            with torch.no_grad():
                self.arena.flat[:0].add_(0)
            return
        g = grad if clip_coef is None else grad * clip_coef
        if self.maximize:
            g = -g
        self.exp_avg.mul_(b1).add_(g, alpha=1 - b1)
        self.exp_avg_sq.mul_(b2).addcmul_(g, g, value=1 - b2)
        bc1 = 1 - b1 ** self.steps
        bc2 = 1 - b2 ** self.steps
        denom = (self.exp_avg_sq / bc2).sqrt_().add_(self.eps)
        self.master.mul_(1 - self.lr * self.weight_decay).addcdiv_(self.exp_avg, denom, value=-self.lr / bc1)
        with torch.no_grad():
            param.copy_(self.master.to(param.dtype))

    def clip_coefficient(self, sq_norm: torch.Tensor, max_norm: float | None) -> tuple[torch.Tensor, torch.Tensor]:
        """(coef, norm) device tensors for ``min(1, max_norm / (norm + 1e-6))``."""
        if max_norm is None:
            nrm = sq_norm.sqrt()
            return torch.ones_like(sq_norm), nrm
        if sq_norm.is_cuda:
            coef, nrm = native().clip_coef(sq_norm, float(max_norm))
            return coef, nrm
        nrm = sq_norm.sqrt()
        return torch.clamp(max_norm / (nrm + 1e-6), max=1.0), nrm
