"""Packed attention: every segment of a pack in one forward and one backward launch (K02-K07, varlen).

A pack holds several segments (trajectories, turns or forest nodes). Segment
``s`` owns the query rows ``[start, start + length)`` of the pack and attends
to its ancestors (K/V chunks of earlier packs, ``past``), to the pack's own
rows named by ``key_ranges`` (forest ancestors inside the pack) and, causally,
to its own rows. The reference runs such packs through a variable-length
flash kernel over a concatenation of every segment's full key chain
(src/thundersync/engine/streaming.py:1653-1836, one backward per pack).

Here the key buffer is ``[unique ancestor chunks | the pack's own rows]``: an
ancestor chunk shared by several segments (a group's prompt) is stored once,
and the backward's dK/dV work items are key tiles with a list of *consumer*
segments, so a shared prompt's gradient is summed over all its readers inside
one CTA (no per-segment copies, no atomics, fixed order). :class:`PackPlan`
holds the work tables the kernels read (layout documented with ``QItem`` and
``KItem`` in the CUDA source); a plan depends only on the pack's segment
layout and which ancestor inputs repeat, so one plan serves every attention
layer of the pack and is cached.
"""

from __future__ import annotations

import math
from collections import OrderedDict
from dataclasses import dataclass
from typing import Any, Sequence

import numpy as np
import torch

from thundersync_b200.ops._ext import native

__all__ = ["PackPlan", "packed_plan", "packed_attention", "packed_attention_reference", "FULL_VIS"]

BM = 128  # query rows per query item (every forward / dQ kernel)
BK = 128  # keys per key item (every dK / dV kernel)
FULL_VIS = -(1 << 30)


@dataclass
class PackPlan:
    t: int  # pack rows (queries and own keys)
    covered: int  # rows [covered, t) belong to no segment (pack padding)
    sp: int  # ancestor rows at the front of the key buffer
    slots: tuple[int, ...]  # per ancestor input position: its unique chunk
    first: tuple[bool, ...]  # per ancestor input position: first occurrence of its chunk
    chunk_rows: tuple[tuple[int, int], ...]  # unique chunk -> (row0, rows) in the key buffer
    qtab: np.ndarray  # [nq, 8] int32
    far: np.ndarray  # [nf, 2] int32
    ktab: np.ndarray  # [nk, 4] int32
    cons: np.ndarray  # [nc, 4] int32
    device_tabs: dict[Any, tuple[torch.Tensor, ...]]

    def tables(self, device: torch.device) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
        """(qtab, far, ktab, cons) as int32 tensors on ``device`` (uploaded once per device)."""
        key = str(device)
        got = self.device_tabs.get(key)
        if got is None:
            host = [torch.from_numpy(np.ascontiguousarray(a).reshape(-1)) for a in
                    (self.qtab, self.far, self.ktab, self.cons)]
            if device.type == "cuda":
                got = tuple(_upload(x, device) for x in host)
            else:
                got = tuple(x.clone() for x in host)
            self.device_tabs[key] = got
        return got


def _upload(x: torch.Tensor, device: torch.device) -> torch.Tensor:
    # a 16-byte aligned device copy (the kernels read the tables as int4); empty tables get one zero entry
    n = max(4, (x.numel() + 3) // 4 * 4)
    pinned = torch.zeros(n, dtype=torch.int32, pin_memory=True)
    pinned[: x.numel()] = x
    out = torch.empty(n, dtype=torch.int32, device=device)
    out.copy_(pinned, non_blocking=True)
    return out[: max(x.numel(), 0)] if x.numel() else out[:0]


def _merge(ranges: list[tuple[int, int]]) -> list[tuple[int, int]]:
    out: list[tuple[int, int]] = []
    for r0, n in ranges:
        if n <= 0:
            continue
        if out and out[-1][0] + out[-1][1] == r0:
            out[-1] = (out[-1][0], out[-1][1] + n)
        else:
            out.append((r0, n))
    return out


def _build(seg_meta: Sequence[tuple[int, int, int, tuple]], slots: Sequence[int], chunk_lens: Sequence[int],
           t: int) -> PackPlan:
    """seg_meta: per segment (start, end, n_past inputs, key_ranges); slots: unique chunk of each ancestor
    input (segments' inputs concatenated in order); chunk_lens: rows of each unique chunk."""
    chunk_rows, r = [], 0
    for n in chunk_lens:
        chunk_rows.append((r, n))
        r += n
    sp = r
    seen: set[int] = set()
    first = []
    for u in slots:
        first.append(u not in seen)
        seen.add(u)
    # ------------------------------------------------------------ query side
    qrows, far_rows = [], []
    users: list[set[int]] = [set() for _ in chunk_lens]  # unique chunk -> segments reading it
    krange_users: list[tuple[int, int, int]] = []  # (a, b, segment) own-row spans read as ancestors
    pi = 0
    covered = 0
    for si, (s0, s1, npast, kranges) in enumerate(seg_meta):
        T = s1 - s0
        covered = max(covered, s1)
        mine = slots[pi:pi + npast]
        pi += npast
        for u in mine:
            users[u].add(si)
        fr = _merge([chunk_rows[u] for u in mine] + [(sp + a, b - a) for a, b in kranges])
        for a, b in kranges:
            krange_users.append((a, b, si))
        far0 = len(far_rows)
        far_rows.extend(fr)
        far_keys = sum(n for _, n in fr)
        for qt in range(0, T, BM):
            work = far_keys + min(T, qt + BM)
            qrows.append((work, [s0 + qt, qt, T, sp + s0, 0, far0, len(fr), 0]))
    qrows.sort(key=lambda x: -x[0])
    qtab = np.array([row for _, row in qrows], dtype=np.int32).reshape(-1, 8)
    far = np.array(far_rows, dtype=np.int32).reshape(-1, 2)
    # ------------------------------------------------------------ key side
    kitems: list[tuple[int, list[int], list[list[int]]]] = []

    def tile_run(row0: int, n: int, consumers_for) -> None:
        for k0 in range(0, n, BK):
            cnt = min(BK, n - k0)
            cons = consumers_for(k0)
            work = sum(max(0, math.ceil((c[1] - max(0, c[2]) // 64 * 64) / 64)) for c in cons)
            kitems.append((work, [row0 + k0, cnt, 0, len(cons)], cons))

    seg_rows = [(s0, s1 - s0) for s0, s1, _, _ in seg_meta]
    # ancestor region: runs of adjacent unique chunks read by the same segments
    u = 0
    while u < len(chunk_lens):
        w = u + 1
        while w < len(chunk_lens) and users[w] == users[u]:
            w += 1
        row0 = chunk_rows[u][0]
        n = sum(chunk_lens[u:w])
        readers = sorted(users[u])
        tile_run(row0, n, lambda k0, rd=readers: [[seg_rows[s][0], seg_rows[s][1], FULL_VIS, 0] for s in rd])
        u = w
    # own region: each segment's rows, cut where forest ancestor spans start or end
    owner = np.full(t, -1, dtype=np.int64)
    for si, (s0, s1, _, _) in enumerate(seg_meta):
        owner[s0:s1] = si
    cuts = {0, t}
    for s0, s1, _, _ in seg_meta:
        cuts.update((s0, s1))
    for a, b, _ in krange_users:
        cuts.update((a, b))
    bounds = sorted(c for c in cuts if 0 <= c <= t)
    for a, b in zip(bounds[:-1], bounds[1:]):
        if b <= a:
            continue
        si = int(owner[a])
        readers = sorted({y for (ka, kb, y) in krange_users if ka <= a and b <= kb})
        if si < 0:
            tile_run(sp + a, b - a, lambda k0: [[seg_rows[y][0], seg_rows[y][1], FULL_VIS, 0] for y in readers])
            continue
        s0 = seg_rows[si][0]

        def cons_own(k0, a=a, s0=s0, si=si, readers=readers):
            c = [[s0, seg_rows[si][1], a - s0 + k0, 0]]
            return c + [[seg_rows[y][0], seg_rows[y][1], FULL_VIS, 0] for y in readers if y != si]

        tile_run(sp + a, b - a, cons_own)
    kitems.sort(key=lambda x: -x[0])
    ktab_rows, cons_rows = [], []
    for _, row, cons in kitems:
        row[2] = len(cons_rows)
        ktab_rows.append(row)
        cons_rows.extend(cons)
    ktab = np.array(ktab_rows, dtype=np.int32).reshape(-1, 4)
    cons = np.array(cons_rows, dtype=np.int32).reshape(-1, 4)
    return PackPlan(t, covered, sp, tuple(slots), tuple(first), tuple(chunk_rows), qtab, far, ktab, cons, {})


_PLANS: "OrderedDict[tuple, PackPlan]" = OrderedDict()
_PLAN_CACHE = 256


def packed_plan(seg_meta: Sequence[tuple[int, int, int, tuple]], past_k: Sequence[torch.Tensor],
                past_v: Sequence[torch.Tensor], t: int) -> PackPlan:
    """The plan of a pack: ``seg_meta`` per segment (start, end, number of ancestor inputs, key_ranges) and
    the segments' ancestor K/V inputs in order (a chunk repeated across segments is the same tensor)."""
    index: dict[tuple, int] = {}
    slots, lens = [], []
    for k, v in zip(past_k, past_v):
        ident = (k.data_ptr(), v.data_ptr(), k.shape[0])
        u = index.get(ident)
        if u is None:
            u = index[ident] = len(lens)
            lens.append(int(k.shape[0]))
        slots.append(u)
    key = (tuple(seg_meta), tuple(slots), tuple(lens), int(t))
    plan = _PLANS.get(key)
    if plan is None:
        plan = _build(seg_meta, slots, lens, t)
        _PLANS[key] = plan
        if len(_PLANS) > _PLAN_CACHE:
            _PLANS.popitem(last=False)
    else:
        _PLANS.move_to_end(key)
    return plan


def unique_chunks(plan: PackPlan, chunks: Sequence[torch.Tensor]) -> list[torch.Tensor]:
    """The first occurrence of each unique chunk, in key-buffer order."""
    return [c for c, f in zip(chunks, plan.first) if f]


def packed_attention_reference(q, kbuf, vbuf, plan: PackPlan, scale):
    """fp32 oracle of the packed kernels over the same key buffer: per segment, its far ranges then its own
    rows with the bottom-right causal mask. Rows outside every segment are zero."""
    from thundersync_b200.ops.attention import attention_reference

    t, hq, d = q.shape
    out = q.new_zeros(t, hq, d)
    lse = torch.zeros(hq, t, dtype=torch.float32, device=q.device)
    done: set[tuple] = set()
    for row in plan.qtab:
        q_row0, q_loc0, T, near_row0, off, far0, nfar, _ = (int(x) for x in row)
        s0 = q_row0 - q_loc0
        if (s0, T) in done:
            continue
        done.add((s0, T))
        ranges = [tuple(int(y) for y in plan.far[far0 + i]) for i in range(nfar)]
        ks = [kbuf[r0:r0 + n] for r0, n in ranges] + [kbuf[near_row0:near_row0 + off + T]]
        vs = [vbuf[r0:r0 + n] for r0, n in ranges] + [vbuf[near_row0:near_row0 + off + T]]
        o, l = attention_reference(q[s0:s0 + T], torch.cat(ks, 0), torch.cat(vs, 0), scale)
        out[s0:s0 + T] = o
        lse[:, s0:s0 + T] = l
    return out, lse


class _PackedAttention(torch.autograd.Function):
    """q [t, Hq, d] and the pack's own k / v [t, Hkv, d] plus the unique ancestor chunks."""

    @staticmethod
    def forward(ctx, q, k_own, v_own, plan, scale, n, *chunks):
        ks, vs = chunks[:n], chunks[n:]
        t, hq, d = q.shape
        kbuf = torch.cat([*ks, k_own], 0) if n else k_own.contiguous()
        vbuf = torch.cat([*vs, v_own], 0) if n else v_own.contiguous()
        q = q.contiguous()
        if q.is_cuda:
            qtab, far, _, _ = plan.tables(q.device)
            out = q.new_empty(t, hq, d)
            _, lse = native().attn_fwd_packed(q, kbuf, vbuf, qtab, far, float(scale), out)
            if plan.covered < t:
                out[plan.covered:].zero_()
                lse[:, plan.covered:].zero_()
        else:
            out, lse = packed_attention_reference(q, kbuf, vbuf, plan, scale)
        ctx.plan, ctx.scale, ctx.n = plan, scale, n
        ctx.lens = [c.shape[0] for c in ks]
        # chunk references, not the concatenated buffer: an event must not keep a copy of its ancestors
        ctx.save_for_backward(q, out, lse, k_own, v_own, *chunks)
        return out

    @staticmethod
    def backward(ctx, do):
        q, out, lse, k_own, v_own, *chunks = ctx.saved_tensors
        plan, n = ctx.plan, ctx.n
        t = q.shape[0]
        kbuf = torch.cat([*chunks[:n], k_own], 0) if n else k_own.contiguous()
        vbuf = torch.cat([*chunks[n:], v_own], 0) if n else v_own.contiguous()
        if q.is_cuda:
            qtab, far, ktab, cons = plan.tables(q.device)
            dq = torch.empty_like(q)
            if plan.covered < t:
                dq[plan.covered:].zero_()
            dq, dk, dv = native().attn_bwd_packed(do.contiguous(), q, kbuf, vbuf, out, lse, qtab, far, ktab, cons,
                                                  float(ctx.scale), dq)
        else:
            with torch.enable_grad():
                q_ = q.detach().requires_grad_(True)
                k_ = kbuf.detach().requires_grad_(True)
                v_ = vbuf.detach().requires_grad_(True)
                o_, _ = packed_attention_reference(q_, k_, v_, plan, ctx.scale)
                dq, dk, dv = torch.autograd.grad(o_, (q_, k_, v_), do)
        sp = plan.sp
        dks = list(torch.split(dk[:sp], ctx.lens, 0)) if n else []
        dvs = list(torch.split(dv[:sp], ctx.lens, 0)) if n else []
        return (dq, dk[sp:], dv[sp:], None, None, None, *dks, *dvs)


def packed_attention(q, k_own, v_own, segs_meta, past_k, past_v, scale=None):
    """Attention of every segment of a pack. ``segs_meta``: per segment (start, end, number of its ancestor
    chunks in ``past_k``/``past_v``, key_ranges); ``past_k``/``past_v``: the segments' ancestor chunks,
    concatenated segment by segment (a chunk shared by several segments appears once per segment)."""
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    plan = packed_plan(segs_meta, past_k, past_v, q.shape[0])
    ks = unique_chunks(plan, past_k)
    vs = unique_chunks(plan, past_v)
    return _PackedAttention.apply(q, k_own, v_own, plan, float(scale), len(ks), *ks, *vs)
