"""Fused QK-norm + RoPE + head split of the QKV projection output.

One pass over ``qkv = x @ [Wq;Wk;Wv]ᵀ`` of shape [T, (Hq + 2·Hkv)·d] produces
contiguous ``q`` [T, Hq, d] and ``k`` [T, Hkv, d] (per-head RMSNorm, then the
rotate-half rotary embedding at the given positions) and ``v`` [T, Hkv, d].
On CUDA the angle ``pos · inv_freq[i]`` is formed in fp32 inside the kernel
and passed to CUDA's ``sincosf``; no cos/sin tables are materialised. The
backward reads ``qkv`` again and recomputes the norm statistics.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops._ext import native
from thundersync_b200.ops.norm import rms_norm_reference


def rope_inv_freq(rotary_dim: int, theta: float, device=None) -> torch.Tensor:
    """fp32 inverse frequencies ``1 / theta^(2i/r)``, i < r/2, r = rotary dims (HF convention)."""
    idx = torch.arange(0, rotary_dim, 2, dtype=torch.int64, device=device).float()
    return 1.0 / (theta ** (idx / rotary_dim))


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def qk_norm_rope_reference(qkv, q_w, k_w, pos, inv_freq, hq, hkv, d, eps, unit_offset=False):
    """Differentiable fp32 oracle of the fused op (rotary over the first 2*len(inv_freq) dims)."""
    t = qkv.shape[0]
    q = qkv[:, : hq * d].reshape(t, hq, d)
    k = qkv[:, hq * d : (hq + hkv) * d].reshape(t, hkv, d)
    v = qkv[:, (hq + hkv) * d :].reshape(t, hkv, d)
    if q_w is not None:
        q = rms_norm_reference(q, q_w, eps, unit_offset)
        k = rms_norm_reference(k, k_w, eps, unit_offset)
    rd = 2 * inv_freq.shape[0]
    freqs = pos.float()[:, None] * inv_freq.float()[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    cos, sin = emb.cos()[:, None, :], emb.sin()[:, None, :]

    def rot(x):
        xr = x[..., :rd].float()
        out = xr * cos + _rotate_half(xr) * sin
        if rd == d:
            return out.to(qkv.dtype)
        return torch.cat((out, x[..., rd:].float()), -1).to(qkv.dtype)

    return rot(q), rot(k), v.contiguous()


ROPE_TABLE_POSITIONS = 65536
_TABLES: dict[tuple, tuple[torch.Tensor, torch.Tensor]] = {}


def rope_tables(inv_freq: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin of ``position * inv_freq`` for positions below ROPE_TABLE_POSITIONS, cached per device.

    The angle is formed in fp32 exactly as the Hugging Face rotary embedding
    forms it, so the kernels read the same cos/sin values that model computes;
    positions past the table fall back to in-kernel sincos.
    """
    key = (inv_freq.device, inv_freq.data_ptr(), inv_freq.numel())
    got = _TABLES.get(key)
    if got is None:
        pos = torch.arange(ROPE_TABLE_POSITIONS, device=inv_freq.device, dtype=torch.float32)
        ang = pos[:, None] * inv_freq.float()[None, :]
        got = (ang.cos().contiguous(), ang.sin().contiguous())
        _TABLES[key] = got
    return got


class _QKNormRope(torch.autograd.Function):
    @staticmethod
    def forward(ctx, qkv, q_w, k_w, pos, inv_freq, hq, hkv, d, eps, unit, k_out=None, v_out=None):
        # k_out / v_out (CUDA): [t, hkv, d] destinations for k and v, e.g. the tail rows of a buffer whose
        # head rows hold the ancestors' keys, so attention reads one contiguous key range without a copy
        ctx.meta = (hq, hkv, d, eps, unit)
        ctx.has_norm = q_w is not None
        if qkv.is_cuda:
            ct, st = rope_tables(inv_freq)
            q, k, v = native().qk_norm_rope_fwd(
                qkv.contiguous(), q_w, k_w, pos.contiguous(), inv_freq.contiguous(), hq, hkv, d, float(eps), bool(unit),
                ct, st, k_out, v_out,
            )
        else:
            with torch.no_grad():
                q, k, v = qk_norm_rope_reference(qkv, q_w, k_w, pos, inv_freq, hq, hkv, d, eps, unit)
        ctx.save_for_backward(qkv, q_w, k_w, pos, inv_freq)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, q_w, k_w, pos, inv_freq = ctx.saved_tensors
        hq, hkv, d, eps, unit = ctx.meta
        t = qkv.shape[0]
        dq = torch.zeros(t, hq, d, dtype=qkv.dtype, device=qkv.device) if dq is None else dq.contiguous()
        dk = torch.zeros(t, hkv, d, dtype=qkv.dtype, device=qkv.device) if dk is None else dk.contiguous()
        dv = torch.zeros(t, hkv, d, dtype=qkv.dtype, device=qkv.device) if dv is None else dv.contiguous()
        s = _sink.active() if ctx.has_norm else None
        acc_q = acc_k = None
        if qkv.is_cuda:
            ct, st = rope_tables(inv_freq)
            # sink-owned norm weights: the kernel's final reduction adds the gradient straight into the sink
            if s is not None:
                if ctx.needs_input_grad[1] and s.owns(q_w) and s.view(q_w).dtype == torch.float32:
                    acc_q = s.view(q_w)
                if ctx.needs_input_grad[2] and s.owns(k_w) and s.view(k_w).dtype == torch.float32:
                    acc_k = s.view(k_w)
            dqkv, dqw, dkw = native().qk_norm_rope_bwd(
                dq, dk, dv, qkv.contiguous(), q_w, k_w, pos.contiguous(), inv_freq.contiguous(),
                hq, hkv, d, float(eps), bool(unit), ct, st, acc_q, acc_k,
                float(s.scale) if s is not None else 1.0,
            )
        else:
            with torch.enable_grad():
                qkv_ = qkv.detach().requires_grad_(True)
                qw_ = None if q_w is None else q_w.detach().requires_grad_(True)
                kw_ = None if k_w is None else k_w.detach().requires_grad_(True)
                outs = qk_norm_rope_reference(qkv_, qw_, kw_, pos, inv_freq, hq, hkv, d, eps, unit)
                ins = [qkv_] + ([qw_, kw_] if qw_ is not None else [])
                grads = torch.autograd.grad(outs, ins, (dq, dk, dv), allow_unused=True)
            dqkv = grads[0]
            dqw = grads[1].float() if qw_ is not None else None
            dkw = grads[2].float() if kw_ is not None else None
        gq = gk = None
        if ctx.has_norm:
            for w, g, idx, acc in ((q_w, dqw, 1, acc_q), (k_w, dkw, 2, acc_k)):
                if not ctx.needs_input_grad[idx]:
                    continue
                if acc is not None:
                    s.deposits += 1
                elif s is not None and s.owns(w):
                    s.add_(w, g)
                elif idx == 1:
                    gq = g.to(w.dtype)
                else:
                    gk = g.to(w.dtype)
        return dqkv, gq, gk, None, None, None, None, None, None, None, None, None


def qk_norm_rope(qkv, q_w, k_w, pos, inv_freq, hq, hkv, d, eps, unit_offset: bool = False):
    """Rotary over the first ``2 * len(inv_freq)`` dims of each head (all dims for Qwen3,
    a quarter for Qwen3.5's partial rotary); ``unit_offset`` selects (1 + w) norms."""
    return _QKNormRope.apply(qkv, q_w, k_w, pos, inv_freq, hq, hkv, d, eps, unit_offset)
