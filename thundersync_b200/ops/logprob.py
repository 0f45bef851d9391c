"""Fused LM head -> log-sum-exp -> gathered log-prob (and entropy) (K01′).

``lm_head_logprob(hidden [N, D], weight [V, D], target [N])`` returns the fp32
log-probability of each target token without materialising the [N, V]
log-softmax. The forward runs over row blocks; the backward recomputes each
block's logits, forms ``dlogits = g·(onehot − softmax)`` (entropy variant:
``−p·(g_lp + g_H·(log p + H)) + g_lp·onehot``) in one native pass, and
produces ``dH`` and the fp32-accumulated ``dW``. Same contract as the
reference's ``_FusedLinearLogprob`` (src/thundersync/accel/fused_logprob.py:61-308).

On CUDA with bf16 operands both passes run as tcgen05 GEMMs whose epilogue
consumes the logits tile straight out of tensor memory: the forward keeps an
online max / sum-of-exp (and sum of exp·x for the entropy) per row and N tile,
reduced by a second small kernel; the backward's epilogue writes bf16
``dlogits`` directly. The fp32 [rows, V] logits never reach HBM.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops._ext import native
from thundersync_b200.ops.gemm import gemm, gemm_accumulate

# Rows per chunk. The backward materialises a chunk's bf16 dlogits ([rows, V]: 622 MB at 2048 rows of a
# 151,936-token vocabulary) and reduce-adds one fp32 [V, D] weight gradient per chunk into the sink (1.2 GB
# at D = 2048, read and written). Larger chunks move fewer sink bytes, but the streamed step keeps most of
# the device busy with retained graphs: 8192-row chunks (a 2.5 GB dlogits buffer) ran the hybrid config
# (32k-token completions) out of memory, so chunks stay at 2048 rows.
DEFAULT_ROWS = 2048
# tcgen05 GEMM with fused log-sum-exp / dlogits epilogues on CUDA bf16 (False: cuBLAS logits + row kernels)
FUSED_TC = True


def _fused_ok(hidden: torch.Tensor, weight: torch.Tensor) -> bool:
    return (FUSED_TC and hidden.is_cuda and hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and hidden.shape[1] % 8 == 0 and weight.shape[0] % 8 == 0 and hidden.is_contiguous()
            and weight.is_contiguous())


def _logits_fp32(h: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if h.is_cuda and h.dtype == torch.bfloat16:
        return gemm(h, w, out_dtype=torch.float32)
    if h.is_cuda and h.dtype == torch.float16:
        return torch.mm(h, w.t(), out_dtype=torch.float32)
    acc = torch.float64 if h.dtype == torch.float64 else torch.float32
    return torch.mm(h.to(acc), w.to(acc).t())


def _stats_ref(logits: torch.Tensor, tgt: torch.Tensor, with_entropy: bool):
    lse = torch.logsumexp(logits, dim=-1)
    lp = logits.gather(-1, tgt[:, None]).squeeze(-1) - lse
    ent = None
    if with_entropy:
        p = torch.exp(logits - lse[:, None])
        ent = lse - (p * logits).sum(-1)
    return lp, lse, ent


def _dlogits_ref(logits, tgt, lse, g_lp, g_ent, ent):
    p = torch.exp(logits - lse[:, None])
    if g_ent is None:
        d = -p * g_lp[:, None]
    else:
        logp = logits - lse[:, None]
        d = -p * (g_lp[:, None] + g_ent[:, None] * (logp + ent[:, None]))
    d.scatter_add_(-1, tgt[:, None], g_lp[:, None].to(d.dtype))
    return d


class _LMHeadLogprob(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, weight, target, rows, with_entropy):
        n = hidden.shape[0]
        lp = torch.empty(n, dtype=torch.float32 if hidden.dtype != torch.float64 else torch.float64,
                         device=hidden.device)
        lse = torch.empty_like(lp)
        ent = torch.empty_like(lp) if with_entropy else None
        fused = _fused_ok(hidden, weight)
        for r0 in range(0, n, rows):
            r1 = min(n, r0 + rows)
            if fused:
                a, b, c = native().lmhead_lse_tc(hidden[r0:r1], weight, target[r0:r1].contiguous(),
                                                 bool(with_entropy))
                lp[r0:r1] = a
                lse[r0:r1] = b
                if with_entropy:
                    ent[r0:r1] = c
                continue
            logits = _logits_fp32(hidden[r0:r1], weight)
            if logits.is_cuda and logits.dtype == torch.float32:
                a, b, c = native().lse_gather(logits, target[r0:r1].contiguous(), bool(with_entropy))
            else:
                a, b, c = _stats_ref(logits, target[r0:r1], with_entropy)
            lp[r0:r1] = a
            lse[r0:r1] = b
            if with_entropy:
                ent[r0:r1] = c
            del logits
        ctx.rows = rows
        ctx.with_entropy = with_entropy
        ctx.save_for_backward(hidden, target, lse, *( [ent] if with_entropy else []))
        ctx.weight = weight
        if with_entropy:
            ctx.mark_non_differentiable(lse)
            return lp, ent
        return lp

    @staticmethod
    def backward(ctx, g_lp, g_ent=None):
        saved = ctx.saved_tensors
        hidden, target, lse = saved[:3]
        ent = saved[3] if ctx.with_entropy else None
        weight = ctx.weight
        n = hidden.shape[0]
        if g_lp is None:
            g_lp = torch.zeros(n, dtype=lse.dtype, device=lse.device)
        g_lp = g_lp.to(lse.dtype).contiguous()
        if g_ent is not None:
            g_ent = g_ent.to(lse.dtype).contiguous()
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        dh = torch.empty_like(hidden) if need_h else None
        s = _sink.active()
        sink_w = need_w and s is not None and s.owns(weight)
        dw_acc = None
        if need_w and not sink_w:
            dw_acc = torch.zeros(weight.shape, dtype=torch.float32 if weight.dtype != torch.float64 else torch.float64,
                                 device=weight.device)
        fused = _fused_ok(hidden, weight)
        for r0 in range(0, n, ctx.rows):
            r1 = min(n, r0 + ctx.rows)
            h = hidden[r0:r1]
            if fused:
                d = native().lmhead_dlogits_tc(
                    h, weight, target[r0:r1].contiguous(), lse[r0:r1].contiguous(), g_lp[r0:r1],
                    None if g_ent is None else g_ent[r0:r1],
                    None if ent is None else ent[r0:r1].contiguous(),
                )
                logits = None
            else:
                logits = _logits_fp32(h, weight)
            if fused:
                pass
            elif logits.is_cuda and logits.dtype == torch.float32:
                d = native().logprob_dlogits(
                    logits, target[r0:r1].contiguous(), lse[r0:r1].contiguous(), g_lp[r0:r1],
                    None if g_ent is None else g_ent[r0:r1],
                    None if ent is None else ent[r0:r1].contiguous(),
                    hidden.dtype == torch.bfloat16,
                )
            else:
                d = _dlogits_ref(logits, target[r0:r1], lse[r0:r1], g_lp[r0:r1],
                                 None if g_ent is None else g_ent[r0:r1],
                                 None if ent is None else ent[r0:r1])
            del logits
            if d.dtype != hidden.dtype and not d.is_cuda:
                d_mm = d.to(hidden.dtype) if hidden.dtype != torch.float64 else d
            else:
                d_mm = d
            if need_h:
                if d_mm.dtype == hidden.dtype:
                    gemm(d_mm, weight, b_t=False, out=dh[r0:r1])
                else:
                    dh[r0:r1] = d_mm.matmul(weight.to(d_mm.dtype)).to(hidden.dtype)
            if need_w:
                if sink_w:
                    s.addmm_(s.view(weight), d_mm, h)
                elif d_mm.is_cuda and d_mm.dtype != dw_acc.dtype:
                    gemm_accumulate(dw_acc, d_mm, h, a_t=True, b_t=False)
                else:
                    dw_acc.addmm_(d_mm.t().to(dw_acc.dtype), h.to(dw_acc.dtype))
        ctx.weight = None
        dw = None if dw_acc is None else dw_acc.to(weight.dtype)
        return dh, dw, None, None, None


def _check(hidden, weight, target):
    if hidden.dim() != 2:
        raise ValueError(f"hidden must be [N, D], got {tuple(hidden.shape)}")
    if target.shape[0] != hidden.shape[0]:
        raise ValueError("target must have one entry per hidden row")
    if weight.shape[1] != hidden.shape[1]:
        raise ValueError(f"weight {tuple(weight.shape)} does not match hidden dim {hidden.shape[1]}")


ROW_MULTIPLE = 128


def _padded(hidden, target):
    """On CUDA, zero-pad the rows to a multiple of ROW_MULTIPLE (the GEMM shapes then repeat)."""
    n = hidden.shape[0]
    pad = (-n) % ROW_MULTIPLE if hidden.is_cuda else 0
    if not pad:
        return hidden, target, n, 0
    return (torch.cat((hidden, hidden.new_zeros(pad, hidden.shape[1]))),
            torch.cat((target, target.new_zeros(pad))), n, pad)


def _row_block(rows: int, cuda: bool) -> int:
    """Rows per LM-head block: positive; on CUDA rounded up to ROW_MULTIPLE (whole GEMM row tiles)."""
    rows = int(rows)
    if rows < 1:
        raise ValueError("the LM-head row block must be positive")
    return -(-rows // ROW_MULTIPLE) * ROW_MULTIPLE if cuda else rows


def lm_head_logprob(hidden, weight, target, *, rows: int = DEFAULT_ROWS):
    """Log-probs of ``target`` under ``hidden @ weight.T``, ``rows`` rows per block: the backward's
    dlogits buffer (and, off the fused path, the logits buffer) holds one block."""
    _check(hidden, weight, target)
    h, t, n, pad = _padded(hidden, target)
    lp = _LMHeadLogprob.apply(h, weight, t, _row_block(rows, h.is_cuda), False)
    return lp[:n] if pad else lp


def lm_head_logprob_entropy(hidden, weight, target, *, rows: int = DEFAULT_ROWS):
    _check(hidden, weight, target)
    h, t, n, pad = _padded(hidden, target)
    lp, ent = _LMHeadLogprob.apply(h, weight, t, _row_block(rows, h.is_cuda), True)
    return (lp[:n], ent[:n]) if pad else (lp, ent)


def naive_logprob(hidden, weight, target):
    """Oracle: materialise full logits and log-softmax."""
    logits = _logits_fp32(hidden, weight)
    return torch.log_softmax(logits, -1).gather(-1, target[:, None]).squeeze(-1)
