"""Log-probabilities through the LM head without materialising ``[N, V]``.

Public names of the reference's fused log-prob module
(src/thundersync/accel/fused_logprob.py:197-388): ``fused_logprob``,
``fused_logprob_entropy``, ``gathered_logprobs`` and ``naive_logprobs``.
They run :mod:`thundersync_b200.ops.logprob` — row blocks of ``h·Wᵀ`` with an
fp32 accumulator, then this package's CUDA log-sum-exp/gather kernel; the
backward recomputes each block and its fused dlogits kernel. ``chunk`` is the
row-block size.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops.logprob import lm_head_logprob, lm_head_logprob_entropy

__all__ = ["fused_logprob", "fused_logprob_entropy", "gathered_logprobs", "naive_logprobs"]


def _validate(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor) -> None:
    if hidden.dim() != 2:
        raise ValueError(f"hidden must be [N, D], got {tuple(hidden.shape)}")
    if target.shape[0] != hidden.shape[0]:
        raise ValueError("target must have one entry per hidden row")
    if weight.shape[1] != hidden.shape[1]:
        raise ValueError(f"weight {tuple(weight.shape)} does not match hidden dim {hidden.shape[1]}")


def fused_logprob(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor, *, chunk: int = 1024):
    """``log π(target | context)`` per row; ``hidden`` [N, D], ``weight`` [V, D], ``target`` [N]."""
    _validate(hidden, weight, target)
    return lm_head_logprob(hidden, weight, target, rows=chunk)


def fused_logprob_entropy(hidden: torch.Tensor, weight: torch.Tensor, target: torch.Tensor, *, chunk: int = 1024):
    """(log-prob, full-vocabulary entropy) per row, both differentiable."""
    _validate(hidden, weight, target)
    return lm_head_logprob_entropy(hidden, weight, target, rows=chunk)


def _acc(dt: torch.dtype) -> torch.dtype:
    return torch.float32 if dt in (torch.bfloat16, torch.float16) else dt


def gathered_logprobs(hidden: torch.Tensor, weight: torch.Tensor, token_ids: torch.Tensor, loss_mask: torch.Tensor,
                      *, chunk: int = 1024) -> torch.Tensor:
    """[N] log-probs aligned with ``token_ids``, zero where ``loss_mask`` is off (position k uses hidden k-1)."""
    n = token_ids.shape[0]
    idx = loss_mask.nonzero(as_tuple=True)[0]
    idx = idx[idx > 0]
    if idx.numel() == 0:
        return torch.zeros(n, dtype=_acc(hidden.dtype), device=hidden.device)
    lp = fused_logprob(hidden[idx - 1], weight, token_ids[idx], chunk=chunk)
    return torch.zeros(n, dtype=lp.dtype, device=lp.device).index_put((idx,), lp)


def naive_logprobs(hidden: torch.Tensor, weight: torch.Tensor, token_ids: torch.Tensor,
                   loss_mask: torch.Tensor) -> torch.Tensor:
    """Oracle: full ``[N, V]`` logits in the accumulator dtype, log-softmax, gather."""
    acc = _acc(hidden.dtype)
    lp = torch.log_softmax(torch.nn.functional.linear(hidden.to(acc), weight.to(acc)), -1)
    out = torch.zeros(token_ids.shape[0], dtype=acc, device=hidden.device)
    idx = loss_mask.nonzero(as_tuple=True)[0]
    idx = idx[idx > 0]
    if idx.numel() == 0:
        return out
    return out.index_put((idx,), lp[idx - 1].gather(-1, token_ids[idx, None]).squeeze(-1))
