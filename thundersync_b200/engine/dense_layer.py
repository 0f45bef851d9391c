"""One autograd node per dense decoder layer (C16, the per-layer executor op).

A Qwen3 decoder layer is eleven ops (norm, fused QKV projection, QK-norm +
RoPE, attention, output projection, residual, norm, fused gate/up, SwiGLU,
down projection, residual). Run as separate autograd nodes, each costs a
Python ``Function.apply`` in the forward and an engine dispatch plus a Python
backward in the backward — for short trajectories that host work, not the
GPU, sets the pace. ``DenseLayer`` runs the same op implementations (their
``forward``/``backward`` static methods, with a lightweight context object)
inside a single autograd node: same kernels, same numerics, same gradient
sink behaviour, one node per layer.

Inputs are the residual stream ``h``, the ancestor K/V chunks of every
segment (gradient channels to earlier segments and prompts) and the layer's
parameters; outputs are the new residual stream and the layer's fresh K and
V for the whole pack (each segment's slice is its state for descendants).
The reference's layer ops play the same role (src/thundersync/engine/
streaming.py:2209-2570, ``_SegLayerCkpt`` and friends).
"""

from __future__ import annotations

import math
from typing import Any

import torch

from thundersync_b200.ops import sink as _sink
from thundersync_b200.ops._ext import native
from thundersync_b200.ops.attention import _ChunkedAttention
from thundersync_b200.ops.linear import _Linear
from thundersync_b200.ops.norm import _RMSNorm
from thundersync_b200.ops.packed_attention import packed_plan, unique_chunks
from thundersync_b200.ops.rope import _QKNormRope, rope_tables
from thundersync_b200.ops.swiglu import _SwiGLU

__all__ = ["DenseLayer", "dense_layer"]

# CUDA single-segment packs: run the layer's forward and backward from C++ (csrc/dense_layer.cpp);
# False keeps the same kernels driven from Python
NATIVE = True
# packs with at least this many rows put their weight-gradient GEMMs on the side stream
SIDE_STREAM_MIN_ROWS = 2048


class _Ctx:
    """The parts of an autograd context the op implementations use."""

    __slots__ = ("needs_input_grad", "saved_tensors", "__dict__")

    def __init__(self, needs: tuple[bool, ...]) -> None:
        self.needs_input_grad = needs
        self.saved_tensors = ()

    def save_for_backward(self, *tensors) -> None:
        self.saved_tensors = tensors


class _Slot:
    """Placeholder for the i-th tensor handed to ``ctx.save_for_backward``."""

    __slots__ = ("i",)

    def __init__(self, i: int) -> None:
        self.i = i


def _stash(ctx) -> None:
    """Move every tensor the layer keeps for its backward (the native path's activations, the inner ops'
    saved tensors) into one ``ctx.save_for_backward`` call, leaving index slots behind. Saved-tensor hooks
    -- activation checkpointing, host offload of checkpoint inputs -- then see all of them."""
    flat: list[torch.Tensor] = []

    def enc(x):
        if isinstance(x, torch.Tensor):
            flat.append(x)
            return _Slot(len(flat) - 1)
        if isinstance(x, _Ctx):
            x.saved_tensors = tuple(enc(t) for t in x.saved_tensors)
            return x
        if isinstance(x, list):
            return [enc(y) for y in x]
        if isinstance(x, tuple) and not isinstance(x, torch.Size):
            return tuple(enc(y) for y in x)
        return x

    ctx.att = enc(getattr(ctx, "att", None))
    ctx.stages = enc(getattr(ctx, "stages", None))
    ctx.save_for_backward(*flat)


def _unstash(ctx) -> None:
    flat = ctx.saved_tensors

    def dec(x):
        if isinstance(x, _Slot):
            return flat[x.i]
        if isinstance(x, _Ctx):
            x.saved_tensors = tuple(dec(t) for t in x.saved_tensors)
            return x
        if isinstance(x, list):
            return [dec(y) for y in x]
        if isinstance(x, tuple) and not isinstance(x, torch.Size):
            return tuple(dec(y) for y in x)
        return x

    ctx.att = dec(ctx.att)
    ctx.stages = dec(ctx.stages)


def _past_grads(plan, lens, buf) -> list:
    """Gradients of the ancestor inputs from the ancestor rows of a key-buffer gradient: one slice per input
    (single segment), or per unique chunk with None for its repeated inputs (packed; autograd sums the
    inputs of one tensor, and a packed chunk's slice already holds every reader's contribution)."""
    if plan is None:
        return list(torch.split(buf, lens, 0)) if lens else []
    rows = plan.chunk_rows
    return [buf[rows[u][0]:rows[u][0] + rows[u][1]] if f else None for u, f in zip(plan.slots, plan.first)]


class DenseLayer(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, pos, inv_freq, meta, *tensors):
        # meta: (hq, hkv, d, eps, scale, segs, n_past, qkv_fused, gu_fused, has_qk_norm)
        hq, hkv, d, eps, scale, segs, n_past, qkv_fused, gu_fused, has_qk = meta
        past = tensors[:n_past]
        p = list(tensors[n_past:])
        ln1, wq, wk, wv = p[0], p[1], p[2], p[3]
        i = 4
        qn = kn = None
        if has_qk:
            qn, kn = p[4], p[5]
            i = 6
        wo, ln2, wg, wu, wd = p[i:i + 5]
        need_w = any(ctx.needs_input_grad[4 + n_past:])
        t = h.shape[0]

        # one segment from row 0 with no own-pack key ranges (a trajectory or prompt pack): on CUDA the
        # ancestors' keys/values and this pack's are laid out in one buffer, the rope kernel writes the
        # pack's rows in place and attention reads / writes every operand where it lives (no concatenation,
        # no zero-filled gradient buffers beyond the padding rows). Any other CUDA pack (several segments,
        # forest key ranges) runs the same way with packed attention: the buffer holds each unique ancestor
        # chunk once and one launch covers every segment.
        fast = (h.is_cuda and len(segs) == 1 and segs[0][0] == 0 and not segs[0][3]
                and segs[0][2] == n_past // 2)
        packed = h.is_cuda and not fast
        plan = packed_plan(segs, past[:n_past // 2], past[n_past // 2:], t) if packed else None
        ctx.fast = fast or packed
        ctx.native = ctx.fast and NATIVE and qkv_fused is not None and gu_fused is not None
        if ctx.fast:
            if plan is None:
                pk, pv = list(past[:n_past // 2]), list(past[n_past // 2:])
                cov = segs[0][1]
            else:
                pk, pv = unique_chunks(plan, past[:n_past // 2]), unique_chunks(plan, past[n_past // 2:])
                cov = plan.covered
            lens = [x.shape[0] for x in pk]
            sp = sum(lens)
        if ctx.native:
            # the whole layer from C++ (same kernels and GEMMs, no per-op Python dispatch)
            ct, st = rope_tables(inv_freq)
            hc = h.contiguous()
            tabs = [] if plan is None else list(plan.tables(h.device)[:2])
            out, k, v, *saved = native().dense_layer_fwd(
                hc, pos, inv_freq, ct, st, ln1, qkv_fused, qn, kn, wo, ln2, gu_fused, wd, pk, pv,
                hq, hkv, d, float(eps), float(scale), int(cov), tabs)
            ctx.att = (hc, pos, inv_freq, ct, st, k, v, list(pk), list(pv), saved, sp, int(cov), lens, plan)
            ctx.params = (ln1, (wq, wk, wv), qn, kn, wo, ln2, (wg, wu), wd, qkv_fused, gu_fused)
            ctx.stages = (None,) * 9
            ctx.set_materialize_grads(False)
            ctx.meta = meta
            ctx.t = t
            ctx.out_shape, ctx.out_dtype, ctx.out_device = out.shape, out.dtype, out.device
            _stash(ctx)
            return out, k, v
        c_n1 = _Ctx((True, need_w, False, False))
        x1 = _RMSNorm.forward(c_n1, h, ln1, eps, False)
        c_qkv = _Ctx((True, False, need_w, need_w, need_w))
        qkv = _Linear.forward(c_qkv, x1, qkv_fused, wq, wk, wv)
        c_rope = _Ctx((True, need_w, need_w) + (False,) * 9)
        if ctx.fast:
            # the pack's own k / v are tensors of their own (descendants keep them as state); the
            # [ancestors | own] buffer attention reads is a temporary, rebuilt in the backward, so no
            # event retains a copy of its ancestors' keys
            q, k, v = _QKNormRope.forward(c_rope, qkv, qn, kn, pos, inv_freq, hq, hkv, d, eps, False)
            kbuf = torch.cat([*pk, k], 0) if pk else k
            vbuf = torch.cat([*pv, v], 0) if pv else v
            o = q.new_empty(t, hq, d)
            if plan is None:
                _, lse = native().attn_fwd_tc(q[:cov], kbuf[:sp + cov], vbuf[:sp + cov], scale, o[:cov])
            else:
                qtab, far, _, _ = plan.tables(h.device)
                _, lse = native().attn_fwd_packed(q, kbuf, vbuf, qtab, far, scale, o)
            del kbuf, vbuf
            if cov < t:  # pack padding rows: no attention output
                o[cov:].zero_()
            ctx.att = (q, k, v, list(pk), list(pv), o, lse, sp, cov, lens, plan)
            c_att = None
            return DenseLayer._forward_tail(ctx, h, o, t, hq, d, eps, need_w, c_n1, c_qkv, c_rope, c_att,
                                            wo, ln2, wg, wu, wd, gu_fused, meta, k, v)
        q, k, v = _QKNormRope.forward(c_rope, qkv, qn, kn, pos, inv_freq, hq, hkv, d, eps, False)
        # attention per segment: [ancestor chunks..., own-pack key ranges..., own slice]
        c_att = []
        outs = []
        pi = 0
        for (s0, s1, npast, kranges) in segs:
            pk = list(past[pi:pi + npast])
            pv = list(past[n_past // 2 + pi:n_past // 2 + pi + npast])
            pi += npast
            ks = pk + [k[a:b] for a, b in kranges] + [k[s0:s1]]
            vs = pv + [v[a:b] for a, b in kranges] + [v[s0:s1]]
            n = len(ks)
            c = _Ctx((True, False, False) + (True,) * (2 * n))
            outs.append(_ChunkedAttention.forward(c, q[s0:s1], scale, n, *ks, *vs))
            c_att.append((c, s0, s1, npast, kranges))
        covered = sum(b - a for a, b, _, _ in segs)
        if covered < t:  # pack padding rows: no attention output
            outs.append(q.new_zeros(t - covered, hq, d))
        o = outs[0] if len(outs) == 1 else torch.cat(outs, 0)
        return DenseLayer._forward_tail(ctx, h, o, t, hq, d, eps, need_w, c_n1, c_qkv, c_rope, c_att,
                                        wo, ln2, wg, wu, wd, gu_fused, meta, k, v)

    @staticmethod
    def _forward_tail(ctx, h, o, t, hq, d, eps, need_w, c_n1, c_qkv, c_rope, c_att, wo, ln2, wg, wu, wd, gu_fused,
                      meta, k, v):
        o = o.reshape(t, hq * d)
        c_o = _Ctx((True, False, need_w))
        h1 = _Linear.forward_residual(c_o, o, None, h, wo)
        c_n2 = _Ctx((True, need_w, False, False))
        x2 = _RMSNorm.forward(c_n2, h1, ln2, eps, False)
        c_gu = _Ctx((True, False, need_w, need_w))
        gu = _Linear.forward(c_gu, x2, gu_fused, wg, wu)
        c_sw = _Ctx((True,))
        a = _SwiGLU.forward(c_sw, gu)
        c_dn = _Ctx((True, False, need_w))
        out = _Linear.forward_residual(c_dn, a, None, h1, wd)
        ctx.stages = (c_n1, c_qkv, c_rope, c_att, c_o, c_n2, c_gu, c_sw, c_dn)
        # K/V outputs that no descendant reads get None gradients, not zero-filled tensors
        ctx.set_materialize_grads(False)
        ctx.meta = meta
        ctx.t = t
        ctx.out_shape, ctx.out_dtype, ctx.out_device = out.shape, out.dtype, out.device
        if not isinstance(getattr(ctx, "att", None), tuple):
            ctx.att = None
        _stash(ctx)
        return out, k, v

    @staticmethod
    def backward(ctx, dout, dk_out, dv_out):
        _unstash(ctx)
        if dout is None:
            dout = torch.zeros(ctx.out_shape, dtype=ctx.out_dtype, device=ctx.out_device)
        if ctx.native:
            return DenseLayer._native_backward(ctx, dout, dk_out, dv_out)
        c_n1, c_qkv, c_rope, c_att, c_o, c_n2, c_gu, c_sw, c_dn = ctx.stages
        hq, hkv, d, eps, scale, segs, n_past, qkv_fused, gu_fused, has_qk = ctx.meta
        t = ctx.t
        # h_out = h1 + down(swiglu(gu(norm2(h1))))
        da, _, gwd = _Linear.backward(c_dn, dout)
        dgu = _SwiGLU.backward(c_sw, da)
        dx2, _, gwg, gwu = _Linear.backward(c_gu, dgu)
        dh1, gln2, _, _ = _RMSNorm.backward_residual(c_n2, dx2, dout)
        # h1 = h + o_proj(o)
        do_, _, gwo = _Linear.backward(c_o, dh1)
        do_ = do_.reshape(t, hq, d)
        if ctx.fast:
            q, k, v, pk, pv, o, lse, sp, cov, lens, plan = ctx.att
            ctx.att = None
            kbuf = torch.cat([*pk, k], 0) if pk else k
            vbuf = torch.cat([*pv, v], 0) if pv else v
            dq = torch.empty_like(q)
            dkbuf = torch.empty_like(kbuf)
            dvbuf = torch.empty_like(vbuf)
            if cov < t:
                dq[cov:].zero_()
            if plan is None:
                if cov < t:
                    dkbuf[sp + cov:].zero_()
                    dvbuf[sp + cov:].zero_()
                native().attn_bwd_tc(do_[:cov].contiguous(), q[:cov], kbuf[:sp + cov], vbuf[:sp + cov], o[:cov],
                                     lse, scale, dq[:cov], dkbuf[:sp + cov], dvbuf[:sp + cov])
            else:
                native().attn_bwd_packed(do_.contiguous(), q, kbuf, vbuf, o, lse, *plan.tables(q.device), scale, dq,
                                         dkbuf, dvbuf)
            dk, dv = dkbuf[sp:], dvbuf[sp:]
            if dk_out is not None:
                dk.add_(dk_out)
            if dv_out is not None:
                dv.add_(dv_out)
            dpast_k = _past_grads(plan, lens, dkbuf[:sp])
            dpast_v = _past_grads(plan, lens, dvbuf[:sp])
            return DenseLayer._finish(ctx, dq, dk, dv, dpast_k, dpast_v, dh1, gln2, gwo, gwg, gwu, gwd)
        covered = sum(s1 - s0 for _, s0, s1, _, _ in c_att)
        single = len(c_att) == 1 and covered == t
        if single and not c_att[0][4]:
            # one segment over the whole pack, no own-pack key ranges: the attention gradients are the outputs
            c, s0, s1, npast, _ = c_att[0]
            g = _ChunkedAttention.backward(c, do_)
            n = npast + 1
            gks, gvs = g[3:3 + n], g[3 + n:3 + 2 * n]
            dk = gks[-1] if dk_out is None else dk_out + gks[-1]
            dv = gvs[-1] if dv_out is None else dv_out + gvs[-1]
            return DenseLayer._finish(ctx, g[0], dk, dv, list(gks[:npast]), list(gvs[:npast]), dh1, gln2, gwo,
                                      gwg, gwu, gwd)
        dq = None if single else torch.zeros(t, hq, d, dtype=do_.dtype, device=do_.device)
        dk = torch.zeros(t, hkv, d, dtype=do_.dtype, device=do_.device) if dk_out is None else dk_out.clone()
        dv = torch.zeros(t, hkv, d, dtype=do_.dtype, device=do_.device) if dv_out is None else dv_out.clone()
        dpast_k: list[Any] = []
        dpast_v: list[Any] = []
        for c, s0, s1, npast, kranges in c_att:
            g = _ChunkedAttention.backward(c, do_[s0:s1])
            n = npast + len(kranges) + 1
            gq = g[0]
            gks = g[3:3 + n]
            gvs = g[3 + n:3 + 2 * n]
            if dq is None:
                dq = gq
            else:
                dq[s0:s1] = gq
            dpast_k.extend(gks[:npast])
            dpast_v.extend(gvs[:npast])
            for j, (a, b) in enumerate(kranges):
                dk[a:b] += gks[npast + j]
                dv[a:b] += gvs[npast + j]
            dk[s0:s1] += gks[-1]
            dv[s0:s1] += gvs[-1]
        return DenseLayer._finish(ctx, dq, dk, dv, dpast_k, dpast_v, dh1, gln2, gwo, gwg, gwu, gwd)

    @staticmethod
    def _native_backward(ctx, dout, dk_out, dv_out):
        hq, hkv, d, eps, scale, segs, n_past, qkv_fused, gu_fused, has_qk = ctx.meta
        h, pos, inv_freq, ct, st, k_own, v_own, pk, pv, saved, sp, cov, lens, plan = ctx.att
        ctx.att = None
        ln1, wqkv_list, qn, kn, wo, ln2, wgu_list, wd, qkv_fused, gu_fused = ctx.params
        ctx.params = None
        need_w = any(ctx.needs_input_grad[4 + n_past:])
        s = _sink.active() if need_w else None
        dev = h.device

        def view(p):
            if s is None or p is None or not s.owns(p):
                return None
            v = s.view(p)
            return v if v.dtype == torch.float32 else None

        def span(ps):
            if s is None or not all(s.owns(p) for p in ps):
                return None
            v = s.span_view(list(ps))
            return v if v is not None and v.dtype == torch.float32 else None

        sinks = [view(ln1), span(wqkv_list), view(qn), view(kn), view(wo), view(ln2), span(wgu_list), view(wd)]
        side = 0
        # short packs are bound by host issue time, where the side stream's extra stream bookkeeping only costs
        if s is not None and _sink.SIDE_STREAM_WEIGHT_GRADS and ctx.t >= SIDE_STREAM_MIN_ROWS:
            side = _sink._side_stream(dev).cuda_stream
            s._side_devices = getattr(s, "_side_devices", set())
            s._side_devices.add(dev)
        res = native().dense_layer_bwd(
            dout, dk_out, dv_out, h, pos, inv_freq, ct, st, ln1, qkv_fused, qn, kn, wo, ln2, gu_fused, wd,
            k_own, v_own, pk, pv, saved, hq, hkv, d, float(eps), float(scale), cov, sp, sinks,
            float(s.scale) if s is not None else 1.0, side, [] if plan is None else list(plan.tables(dev)))
        dh, dkp, dvp, g_ln1, g_qkv, g_qn, g_kn, g_o, g_ln2, g_gu, g_d = res
        if s is not None:
            s.deposits += sum(1 for x in sinks if x is not None)
        dpast_k = _past_grads(plan, lens, dkp)
        dpast_v = _past_grads(plan, lens, dvp)

        def cast(g, p):
            return None if g is None or p is None else g.to(p.dtype)

        def split(g, ps):
            if g is None:
                return [None] * len(ps)
            out, r0 = [], 0
            for p in ps:
                out.append(g[r0:r0 + p.shape[0]].to(p.dtype))
                r0 += p.shape[0]
            return out

        gq, gk, gv = split(g_qkv, wqkv_list)
        gg, gu = split(g_gu, wgu_list)
        params = [cast(g_ln1, ln1), gq, gk, gv] + ([cast(g_qn, qn), cast(g_kn, kn)] if has_qk else [])
        params += [cast(g_o, wo), cast(g_ln2, ln2), gg, gu, cast(g_d, wd)]
        return (dh, None, None, None, *dpast_k, *dpast_v, *params)

    @staticmethod
    def _finish(ctx, dq, dk, dv, dpast_k, dpast_v, dh1, gln2, gwo, gwg, gwu, gwd):
        c_n1, c_qkv, c_rope = ctx.stages[:3]
        has_qk = ctx.meta[9]
        dqkv, gqn, gkn, *_ = _QKNormRope.backward(c_rope, dq, dk, dv)
        dx1, _, gwq, gwk, gwv = _Linear.backward(c_qkv, dqkv)
        dh, gln1, _, _ = _RMSNorm.backward_residual(c_n1, dx1, dh1)
        ctx.stages = None
        params = [gln1, gwq, gwk, gwv] + ([gqn, gkn] if has_qk else []) + [gwo, gln2, gwg, gwu, gwd]
        return (dh, None, None, None, *dpast_k, *dpast_v, *params)


def dense_layer(ex, i: int, h: torch.Tensor, pos: torch.Tensor, segs) -> tuple[torch.Tensor, list]:
    """Run dense attention layer ``i`` of executor ``ex`` as one autograd node; returns (h, per-seg (k, v))."""
    spec = ex.spec
    arena = ex.arena
    # the layer's parameter list, fused weight views and scalars do not change between calls (the same
    # parameter objects, the same arena): build them once per layer
    cache = ex.__dict__.setdefault("_dense_static", {})
    layer = ex.model.model.layers[i]
    st = cache.get(i)
    if st is None or st[0] is not arena or st[1] is not layer.input_layernorm.weight:
        sa, mlp = layer.self_attn, layer.mlp
        qn = getattr(sa, "q_norm", None)
        kn = getattr(sa, "k_norm", None)
        has_qk = qn is not None
        weights_qkv = [sa.q_proj.weight, sa.k_proj.weight, sa.v_proj.weight]
        weights_gu = [mlp.gate_proj.weight, mlp.up_proj.weight]
        qkv_fused = arena.fused_weight(weights_qkv) if arena is not None else None
        gu_fused = arena.fused_weight(weights_gu) if arena is not None else None
        eps = getattr(layer.input_layernorm, "variance_epsilon", None) or spec.eps
        params = [layer.input_layernorm.weight, *weights_qkv]
        if has_qk:
            params += [qn.weight, kn.weight]
        params += [sa.o_proj.weight, layer.post_attention_layernorm.weight, *weights_gu, mlp.down_proj.weight]
        st = (arena, layer.input_layernorm.weight, tuple(params), qkv_fused, gu_fused, eps, has_qk)
        cache[i] = st
    _, _, params, qkv_fused, gu_fused, eps, has_qk = st
    past_k, past_v, seg_meta = [], [], []
    for seg in segs:
        ks, vs = seg.past[i] if seg.past and seg.past[i] is not None else ([], [])
        past_k.extend(ks)
        past_v.extend(vs)
        seg_meta.append((seg.start, seg.start + seg.length, len(ks), tuple(seg.key_ranges)))
    meta = (spec.n_heads, spec.n_kv, spec.head_dim, eps, 1.0 / math.sqrt(spec.head_dim), tuple(seg_meta),
            len(past_k) + len(past_v), qkv_fused, gu_fused, has_qk)
    out, k, v = DenseLayer.apply(h, pos, ex.inv_freq(h.device), meta, *past_k, *past_v, *params)
    new_state = [(k[s.start:s.start + s.length], v[s.start:s.start + s.length]) for s in segs]
    return out, new_state
