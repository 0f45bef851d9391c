"""Gated DeltaNet sequence mixing: causal depthwise conv1d (K08′) and the gated delta rule (K09′).

``causal_conv1d_silu(x, weight, tail)``
    x [T, C], weight [C, K], tail [K-1, C] (the previous K-1 pre-conv inputs
    of this channel stream, zeros at a root). Returns ``silu(conv(x))`` [T, C]
    and the new tail (the last K-1 rows of ``[tail; x]``). The tail is a
    gradient channel, exactly like ancestor K/V for attention.

``gated_delta_rule(q, k, v, g, beta, state)``
    q, k [T, H, dk], v [T, H, dv], g and beta [T, H] (g = log decay), state
    [H, dk, dv] fp32 or None. q and k are L2-normalised inside (eps 1e-6) and
    q is scaled by dk^-1/2; per head and token::

        S <- exp(g_t) S
        S <- S + k_t (beta_t (v_t - S^T k_t))^T
        o_t = S^T q_t

    Returns o [T, H, dv] and the final state (fp32). The initial state and
    the final state are both gradient channels (``dh0`` / ``dht``).

Both ops run this package's CUDA kernels on CUDA and the exact recurrences
in fp32 torch on CPU (reference: the HF ``torch_causal_conv1d`` /
``torch_recurrent_gated_delta_rule`` semantics the reference calls at
src/thundersync/engine/streaming.py:1966-2026).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from thundersync_b200.ops._ext import native

__all__ = ["causal_conv1d_silu", "gated_delta_rule", "gated_delta_rule_reference", "causal_conv1d_reference"]


# ---------------------------------------------------------------------------- conv1d
def causal_conv1d_reference(x: torch.Tensor, weight: torch.Tensor, tail: torch.Tensor | None):
    k = weight.shape[1]
    t, c = x.shape
    if tail is None:
        tail = x.new_zeros(k - 1, c)
    full = torch.cat((tail.to(x.dtype), x), 0)  # [K-1+T, C]
    y = F.conv1d(full.t()[None].float(), weight.float()[:, None, :], groups=c)[0].t()  # [T, C]
    out = F.silu(y).to(x.dtype)
    return out, full[-(k - 1):] if k > 1 else full[:0]


class _Conv1d(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, weight, tail):
        ctx.save_for_backward(x, weight, tail)
        if x.is_cuda:
            y, new_tail = native().conv1d_silu_fwd(x.contiguous(), weight.contiguous(), tail.contiguous())
        else:
            with torch.no_grad():
                y, new_tail = causal_conv1d_reference(x, weight, tail)
        return y, new_tail

    @staticmethod
    def backward(ctx, dy, dtail_out):
        x, weight, tail = ctx.saved_tensors
        if dy is None:
            dy = torch.zeros_like(x)
        if dtail_out is None:
            dtail_out = torch.zeros_like(tail)
        if x.is_cuda:
            dx, dw, dtail = native().conv1d_silu_bwd(dy.contiguous(), dtail_out.contiguous(), x.contiguous(),
                                                     weight.contiguous(), tail.contiguous())
            dw = dw.to(weight.dtype)
        else:
            with torch.enable_grad():
                x_ = x.detach().requires_grad_(True)
                w_ = weight.detach().requires_grad_(True)
                t_ = tail.detach().requires_grad_(True)
                y, nt = causal_conv1d_reference(x_, w_, t_)
                dx, dw, dtail = torch.autograd.grad((y, nt), (x_, w_, t_), (dy, dtail_out), allow_unused=True)
            dtail = torch.zeros_like(tail) if dtail is None else dtail
        return dx, dw, dtail


def causal_conv1d_silu(x: torch.Tensor, weight: torch.Tensor, tail: torch.Tensor | None):
    """(silu(causal depthwise conv), new tail); ``weight`` is [C, K] (the conv1d weight squeezed)."""
    if tail is None:
        tail = x.new_zeros(weight.shape[1] - 1, x.shape[1])
    return _Conv1d.apply(x, weight, tail)


# ---------------------------------------------------------------------------- delta rule
def _l2n(x: torch.Tensor) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + 1e-6)


def gated_delta_rule_reference(q, k, v, g, beta, state=None):
    """Exact recurrence in fp32 (differentiable); [T,H,d] layout."""
    t, h, dk = q.shape
    dv = v.shape[-1]
    qf = _l2n(q.float()) * dk ** -0.5
    kf = _l2n(k.float())
    vf, gf, bf = v.float(), g.float(), beta.float()
    s = torch.zeros(h, dk, dv, dtype=torch.float32, device=q.device) if state is None else state.float()
    outs = []
    for i in range(t):
        s = s * gf[i].exp()[:, None, None]
        kv = torch.einsum("hk,hkv->hv", kf[i], s)
        delta = (vf[i] - kv) * bf[i][:, None]
        s = s + kf[i][:, :, None] * delta[:, None, :]
        outs.append(torch.einsum("hk,hkv->hv", qf[i], s))
    o = torch.stack(outs, 0) if outs else vf.new_zeros(0, h, dv)
    return o.to(q.dtype), s


# CUDA, dk = dv = 128: the chunked WY-form kernels (serial over 64-token chunks); otherwise the
# token-recurrent kernels
CHUNKED = True


def _chunked_ok(q, v) -> bool:
    return CHUNKED and q.is_cuda and q.shape[-1] == 128 and v.shape[-1] == 128 and q.dtype == torch.bfloat16


class _GDN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, state):
        ctx.chunked = _chunked_ok(q, v)
        if ctx.chunked:
            o, final, *saved = native().gdn_chunk_fwd(
                q.contiguous(), k.contiguous(), v.contiguous(), g.float().contiguous(), beta.float().contiguous(),
                state.float().contiguous())
            ctx.save_for_backward(q, k, v, g, beta, state, *saved)
        elif q.is_cuda:
            o, final, ckpt = native().gdn_fwd(q.contiguous(), k.contiguous(), v.contiguous(), g.float().contiguous(),
                                              beta.float().contiguous(), state.contiguous())
            ctx.save_for_backward(q, k, v, g, beta, state, ckpt)
        else:
            with torch.no_grad():
                o, final = gated_delta_rule_reference(q, k, v, g, beta, state)
            ctx.save_for_backward(q, k, v, g, beta, state)
        return o, final

    @staticmethod
    def backward(ctx, do, dfinal):
        saved = ctx.saved_tensors
        q, k, v, g, beta, state = saved[:6]
        if do is None:
            do = torch.zeros(v.shape, dtype=v.dtype, device=v.device)
        if dfinal is None:
            dfinal = torch.zeros_like(state)
        if ctx.chunked:
            dq, dk, dv, dg, dbeta, dstate = native().gdn_chunk_bwd(
                do.to(q.dtype).contiguous(), dfinal.float().contiguous(), q.contiguous(), k.contiguous(),
                v.contiguous(), g.float().contiguous(), beta.float().contiguous(), *saved[6:])
            return dq, dk, dv, dg.to(g.dtype), dbeta.to(beta.dtype), dstate.to(state.dtype)
        if q.is_cuda:
            ckpt = saved[6]
            dq, dk, dv, dg, dbeta, dstate = native().gdn_bwd(
                do.contiguous(), dfinal.float().contiguous(), q.contiguous(), k.contiguous(), v.contiguous(),
                g.float().contiguous(), beta.float().contiguous(), ckpt)
            return dq, dk, dv, dg.to(g.dtype), dbeta.to(beta.dtype), dstate
        with torch.enable_grad():
            ins = [x.detach().requires_grad_(True) for x in (q, k, v, g, beta, state)]
            o, fin = gated_delta_rule_reference(*ins)
            grads = torch.autograd.grad((o, fin), ins, (do, dfinal), allow_unused=True)
        return tuple(torch.zeros_like(x) if gr is None else gr for x, gr in zip(ins, grads))


def gated_delta_rule(q, k, v, g, beta, state=None):
    if state is None:
        state = torch.zeros(q.shape[1], q.shape[2], v.shape[2], dtype=torch.float32, device=q.device)
    return _GDN.apply(q, k, v, g, beta, state)
