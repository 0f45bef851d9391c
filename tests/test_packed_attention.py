"""Packed (variable-length) attention: the work tables and the op against per-segment attention.

CPU: the query-side tables (far ranges + near range) and the key-side tables (key tiles + consumers) must
describe the same query/key visibility as per-segment bottom-right causal attention over each segment's
chain, every key row must sit in exactly one key item, and the op's forward/backward (fp64 oracle path)
must equal per-segment ``chunked_attention``. GPU: the tcgen05 packed kernels against the fp32 oracle.
"""

from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from thundersync_b200.ops.attention import attention_reference, chunked_attention
from thundersync_b200.ops.packed_attention import BK, BM, packed_attention, packed_plan


def _layout(rng: random.Random, n_seg: int, *, forest: bool, pad: int, dtype=torch.float64, device="cpu",
            hkv=2, d=16, long=False):
    """Random pack: shared prompt chunks, per-segment extra chunks, optional in-pack ancestor spans."""
    lens = [rng.randint(1, 300 if long else 150) for _ in range(n_seg)]
    prompts = [torch.randn(rng.randint(1, 200), hkv, d, dtype=dtype, device=device) for _ in range(2)]
    pv = [torch.randn_like(p) for p in prompts]
    meta, pk, pvv, chains = [], [], [], []
    s0 = 0
    for i, n in enumerate(lens):
        mine_k, mine_v = [], []
        if rng.random() < 0.8:
            j = rng.randrange(2)
            mine_k.append(prompts[j])
            mine_v.append(pv[j])
        if rng.random() < 0.4:
            extra = torch.randn(rng.randint(1, 130), hkv, d, dtype=dtype, device=device)
            mine_k.append(extra)
            mine_v.append(torch.randn_like(extra))
        kr = ()
        if forest and i > 0 and rng.random() < 0.6:
            a = rng.randrange(0, s0)
            b = rng.randint(a + 1, s0)
            kr = ((a, b),)
        meta.append((s0, s0 + n, len(mine_k), kr))
        pk += mine_k
        pvv += mine_v
        chains.append((mine_k, mine_v))
        s0 += n
    t = s0 + pad
    return meta, pk, pvv, chains, t


def _visibility_from_q(plan) -> set:
    vis = set()
    for row in plan.qtab:
        q_row0, q_loc0, T, near_row0, off, far0, nfar, _ = (int(x) for x in row)
        for r in range(BM):
            qi = q_loc0 + r
            if qi >= T:
                break
            for f in range(nfar):
                r0, n = (int(x) for x in plan.far[far0 + f])
                vis.update((q_row0 + r, r0 + j) for j in range(n))
            for b in range(off + T):
                if b <= qi + off:
                    vis.add((q_row0 + r, near_row0 + b))
    return vis


def _visibility_from_k(plan, n_rows: int) -> set:
    vis = set()
    owned = np.zeros(n_rows, dtype=np.int64)
    for k_row0, cnt, c0, nc in plan.ktab:
        assert 0 < cnt <= BK
        owned[k_row0:k_row0 + cnt] += 1
        for c in range(nc):
            q_row0, T, vis_base, _ = (int(x) for x in plan.cons[c0 + c])
            for r in range(cnt):
                for i in range(max(0, vis_base + r), T):
                    vis.add((q_row0 + i, int(k_row0) + r))
    assert (owned == 1).all(), "every key row belongs to exactly one key item"
    return vis


@pytest.mark.parametrize("seed", range(6))
def test_plan_tables_agree(seed):
    rng = random.Random(seed)
    meta, pk, pv, _, t = _layout(rng, rng.randint(1, 6), forest=seed % 2 == 1, pad=rng.choice([0, 7]))
    plan = packed_plan(meta, pk, pv, t)
    assert _visibility_from_q(plan) == _visibility_from_k(plan, plan.sp + t)
    # no ancestor chunk is stored twice
    assert len(plan.chunk_rows) == len({id(x) for x in pk})


@pytest.mark.parametrize("seed", range(4))
def test_packed_matches_per_segment(seed):
    rng = random.Random(100 + seed)
    torch.manual_seed(seed)
    hq, hkv, d = 4, 2, 16
    meta, pk, pv, chains, t = _layout(rng, rng.randint(1, 5), forest=seed >= 2, pad=3 * (seed % 2))
    leaves = [x.requires_grad_(True) for x in {id(x): x for x in pk + pv}.values()]
    q = torch.randn(t, hq, d, dtype=torch.float64, requires_grad=True)
    k = torch.randn(t, hkv, d, dtype=torch.float64, requires_grad=True)
    v = torch.randn(t, hkv, d, dtype=torch.float64, requires_grad=True)
    out = packed_attention(q, k, v, meta, pk, pv)
    ref = []
    for (s0, s1, _, kr), (ck, cv) in zip(meta, chains):
        ks = list(ck) + [k[a:b] for a, b in kr] + [k[s0:s1]]
        vs = list(cv) + [v[a:b] for a, b in kr] + [v[s0:s1]]
        ref.append(chunked_attention(q[s0:s1], ks, vs))
    covered = meta[-1][1]
    if covered < t:
        ref.append(q.new_zeros(t - covered, hq, d))
    ref = torch.cat(ref, 0)
    torch.testing.assert_close(out, ref, rtol=1e-10, atol=1e-10)
    g = torch.randn_like(out)
    inputs = [q, k, v, *leaves]
    ga = torch.autograd.grad(out, inputs, g, allow_unused=True)
    gb = torch.autograd.grad(ref, inputs, g, allow_unused=True)
    for a, b in zip(ga, gb):
        if a is None or b is None:
            assert a is None and b is None
            continue
        torch.testing.assert_close(a, b, rtol=1e-9, atol=1e-9)


@pytest.mark.gpu
@pytest.mark.parametrize("d", [64, 128, 256])
@pytest.mark.parametrize("seed", [0, 1])
def test_packed_kernels_match_fp32(d, seed):
    """tcgen05 packed forward/backward over a random pack (shared prompts, in-pack ancestors, padding) against
    the fp32 per-segment oracle."""
    dev = torch.device("cuda")
    rng = random.Random(1000 * d + seed)
    torch.manual_seed(seed)
    hq, hkv = 8, 2
    meta, pk, pv, chains, t = _layout(rng, rng.randint(2, 6), forest=seed == 1, pad=5, dtype=torch.bfloat16,
                                      device=dev, hkv=hkv, d=d, long=True)
    leaves = list({id(x): x for x in pk + pv}.values())
    for x in leaves:
        x.requires_grad_(True)
    q = torch.randn(t, hq, d, dtype=torch.bfloat16, device=dev, requires_grad=True)
    k = torch.randn(t, hkv, d, dtype=torch.bfloat16, device=dev, requires_grad=True)
    v = torch.randn(t, hkv, d, dtype=torch.bfloat16, device=dev, requires_grad=True)
    out = packed_attention(q, k, v, meta, pk, pv)
    g = torch.randn_like(out)
    ga = torch.autograd.grad(out, [q, k, v, *leaves], g)

    def f32(x):
        return x.detach().float().requires_grad_(True)

    qf, kf, vf = f32(q), f32(k), f32(v)
    lf = {id(x): f32(x) for x in leaves}
    ref = []
    for (s0, s1, _, kr), (ck, cv) in zip(meta, chains):
        ks = [lf[id(x)] for x in ck] + [kf[a:b] for a, b in kr] + [kf[s0:s1]]
        vs = [lf[id(x)] for x in cv] + [vf[a:b] for a, b in kr] + [vf[s0:s1]]
        o, _ = attention_reference(qf[s0:s1], torch.cat(ks), torch.cat(vs), 1.0 / d ** 0.5)
        ref.append(o.float() if o.dtype == torch.float32 else o)
    covered = meta[-1][1]
    ref.append(qf.new_zeros(t - covered, hq, d))
    ref = torch.cat(ref, 0)
    gb = torch.autograd.grad(ref, [qf, kf, vf, *[lf[id(x)] for x in leaves]], g.float())

    def rel(a, b):
        return float((a.float() - b).norm() / b.norm().clamp_min(1e-12))

    assert rel(out, ref) < 2e-2
    for a, b in zip(ga, gb):
        assert rel(a, b) < 3e-2
    assert out[covered:].abs().max().item() == 0


def test_plan_is_cached_per_layout_and_repeat_pattern():
    """One plan per (segment layout, which ancestor inputs repeat, chunk lengths): every attention layer of a
    pack reuses it, and a different sharing pattern gets its own tables."""
    a = torch.zeros(7, 2, 16)
    b = torch.zeros(7, 2, 16)
    meta = ((0, 5, 1, ()), (5, 9, 1, ()))
    shared = packed_plan(meta, [a, a], [a, a], 12)
    again = packed_plan(meta, [b, b], [b, b], 12)  # another layer's tensors, same sharing pattern
    distinct = packed_plan(meta, [a, b], [a, b], 12)
    assert shared is again
    assert distinct is not shared
    assert len(shared.chunk_rows) == 1 and len(distinct.chunk_rows) == 2
    assert shared.first == (True, False) and distinct.first == (True, True)


def test_oneshot_threshold_scales_with_world():
    from thundersync_b200.parallel.symm import ONESHOT_MAX_ELEMS, oneshot_max_elems

    assert oneshot_max_elems(2) == ONESHOT_MAX_ELEMS == (16 << 20) // 4
    assert oneshot_max_elems(8) * 4 == oneshot_max_elems(2)
