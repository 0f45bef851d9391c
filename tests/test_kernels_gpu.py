"""Native sm_100a kernels vs plain-torch fp32 references of the same ops."""

from __future__ import annotations

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _rel(a, b):
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-12))


def test_extension_loaded_from_tree():
    from thundersync_b200.ops import _ext

    assert _ext.available()
    assert "thundersync_b200" in _ext.so_path()


@pytest.mark.parametrize("rows,h", [(300, 2048), (17, 64), (1000, 2560), (5, 4096)])
def test_rms_norm(rows, h):
    from thundersync_b200.ops.norm import rms_norm, rms_norm_reference

    torch.manual_seed(0)
    x = torch.randn(rows, h, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (1 + 0.1 * torch.randn(h, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    y = rms_norm(x, w, 1e-6)
    dy = torch.randn_like(y)
    gx, gw = torch.autograd.grad(y, (x, w), dy)
    xr = x.detach().float().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = rms_norm_reference(xr, wr, 1e-6)
    gxr, gwr = torch.autograd.grad(yr, (xr, wr), dy.float())
    torch.testing.assert_close(y.float(), yr, atol=3e-2, rtol=2e-2)
    assert _rel(gx, gxr) < 1e-2
    assert _rel(gw, gwr) < 1e-2
    # deterministic weight gradient
    gx2, gw2 = torch.autograd.grad(rms_norm(x, w, 1e-6), (x, w), dy)
    assert torch.equal(gw, gw2)
    # residual-branch gradient added inside the kernel before the single rounding of dx
    from thundersync_b200.ops._ext import native

    _, rstd = native().rms_norm_fwd(x.detach(), w.detach(), 1e-6, False)
    dres = torch.randn_like(dy)
    dx_r, dw_r = native().rms_norm_bwd(dy, x.detach(), w.detach(), rstd, False, dres)
    torch.testing.assert_close(dx_r.float(), (gxr + dres.float()), atol=2e-2, rtol=1e-2)
    assert torch.equal(dw_r, native().rms_norm_bwd(dy, x.detach(), w.detach(), rstd, False)[1])


@pytest.mark.parametrize("d,hq,hkv,norm", [(128, 4, 2, True), (64, 8, 8, True), (128, 2, 1, False), (256, 4, 1, True)])
def test_qk_norm_rope(d, hq, hkv, norm):
    from thundersync_b200.ops.rope import qk_norm_rope, qk_norm_rope_reference, rope_inv_freq

    torch.manual_seed(1)
    t = 77
    qkv = torch.randn(t, (hq + 2 * hkv) * d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    qw = (1 + 0.1 * torch.randn(d, device=DEV)).to(torch.bfloat16).requires_grad_(True) if norm else None
    kw = (1 + 0.1 * torch.randn(d, device=DEV)).to(torch.bfloat16).requires_grad_(True) if norm else None
    pos = torch.arange(1000, 1000 + t, device=DEV)
    inv = rope_inv_freq(d, 1e6, DEV)
    outs = qk_norm_rope(qkv, qw, kw, pos, inv, hq, hkv, d, 1e-6)
    grads_out = [torch.randn_like(o) for o in outs]
    ins = [qkv] + ([qw, kw] if norm else [])
    g = torch.autograd.grad(outs, ins, grads_out)
    ref_ins = [i.detach().float().requires_grad_(True) for i in ins]
    r = qk_norm_rope_reference(ref_ins[0], ref_ins[1] if norm else None, ref_ins[2] if norm else None,
                               pos, inv, hq, hkv, d, 1e-6)
    gr = torch.autograd.grad(r, ref_ins, [x.float() for x in grads_out])
    for a, b in zip(outs, r):
        torch.testing.assert_close(a.float(), b, atol=3e-2, rtol=2e-2)
    for a, b in zip(g, gr):
        assert _rel(a, b) < 1.5e-2


def test_swiglu():
    from thundersync_b200.ops.swiglu import swiglu, swiglu_reference

    torch.manual_seed(2)
    gu = torch.randn(123, 2 * 6144, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    a = swiglu(gu)
    da = torch.randn_like(a)
    (g,) = torch.autograd.grad(a, gu, da)
    gur = gu.detach().float().requires_grad_(True)
    ar = swiglu_reference(gur)
    (gr,) = torch.autograd.grad(ar, gur, da.float())
    torch.testing.assert_close(a.float(), ar, atol=2e-2, rtol=2e-2)
    assert _rel(g, gr) < 1e-2


ATTN_CASES = [
    (64, 64, 4, 2, 128),
    (130, 300, 4, 2, 256),
    (257, 257, 2, 1, 256),
    (100, 612, 8, 2, 128),
    (1, 300, 4, 4, 64),
    (257, 257, 2, 1, 64),
    (513, 1025, 16, 8, 128),
    (130, 130, 4, 1, 128),
]


@pytest.mark.parametrize("t,s,hq,hkv,d", ATTN_CASES)
def test_attention(t, s, hq, hkv, d):
    from thundersync_b200.ops.attention import attention_reference, chunked_attention

    torch.manual_seed(3)
    q = torch.randn(t, hq, d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    # ancestors + own chunk
    split = s - t
    kc = [k[:split], k[split:]] if split > 0 else [k]
    vc = [v[:split], v[split:]] if split > 0 else [v]
    o = chunked_attention(q, kc, vc)
    do = torch.randn_like(o)
    gq, gk, gv = torch.autograd.grad(o, (q, k, v), do)
    qr, kr, vr = (x.detach().float().requires_grad_(True) for x in (q, k, v))
    orf, _ = attention_reference(qr, kr, vr, 1 / math.sqrt(d))
    gqr, gkr, gvr = torch.autograd.grad(orf, (qr, kr, vr), do.float())
    torch.testing.assert_close(o.float(), orf, atol=2e-2, rtol=2e-2)
    assert _rel(gq, gqr) < 2e-2
    assert _rel(gk, gkr) < 2e-2
    assert _rel(gv, gvr) < 2e-2
    # determinism of the backward
    gq2, gk2, gv2 = torch.autograd.grad(chunked_attention(q, kc, vc), (q, k, v), do)
    assert torch.equal(gq, gq2) and torch.equal(gk, gk2) and torch.equal(gv, gv2)


@pytest.mark.parametrize("entropy", [False, True])
def test_lm_head_logprob(entropy):
    from thundersync_b200.ops.logprob import lm_head_logprob, lm_head_logprob_entropy

    torch.manual_seed(4)
    n, dmod, vocab = 300, 256, 5003
    h = (0.5 * torch.randn(n, dmod, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    w = (0.5 * torch.randn(vocab, dmod, device=DEV)).to(torch.bfloat16).requires_grad_(True)
    tgt = torch.randint(0, vocab, (n,), device=DEV)
    hr, wr = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    logits = hr @ wr.t()
    lsm = torch.log_softmax(logits, -1)
    lpr = lsm.gather(-1, tgt[:, None]).squeeze(-1)
    if entropy:
        lp, ent = lm_head_logprob_entropy(h, w, tgt, rows=128)
        entr = -(lsm.exp() * lsm).sum(-1)
        torch.testing.assert_close(ent, entr, atol=2e-3, rtol=2e-3)
        go, ge = torch.randn_like(lp), torch.randn_like(ent)
        g = torch.autograd.grad((lp, ent), (h, w), (go, ge))
        gr = torch.autograd.grad((lpr, entr), (hr, wr), (go, ge))
    else:
        lp = lm_head_logprob(h, w, tgt, rows=128)
        go = torch.randn_like(lp)
        g = torch.autograd.grad(lp, (h, w), go)
        gr = torch.autograd.grad(lpr, (hr, wr), go)
    torch.testing.assert_close(lp, lpr, atol=2e-3, rtol=2e-3)
    assert _rel(g[0], gr[0]) < 2e-2
    assert _rel(g[1], gr[1]) < 2e-2


@pytest.mark.parametrize("entropy", [False, True])
@pytest.mark.parametrize("n,dmod,vocab", [(300, 256, 5008), (1000, 2048, 151936)])
def test_lm_head_fused_tcgen05(entropy, n, dmod, vocab):
    """The tcgen05 LSE/dlogits epilogues against an fp32 PyTorch reference and the unfused path."""
    from thundersync_b200.ops import logprob as L

    assert L._fused_ok(torch.empty(1, dmod, device=DEV, dtype=torch.bfloat16),
                       torch.empty(vocab, dmod, device=DEV, dtype=torch.bfloat16))
    torch.manual_seed(14)
    h = (0.5 * torch.randn(n, dmod, device=DEV) / dmod ** 0.25).to(torch.bfloat16).requires_grad_(True)
    w = (0.5 * torch.randn(vocab, dmod, device=DEV) / dmod ** 0.25).to(torch.bfloat16).requires_grad_(True)
    tgt = torch.randint(0, vocab, (n,), device=DEV)
    hr, wr = h.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    lsm = torch.log_softmax(hr @ wr.t(), -1)
    lpr = lsm.gather(-1, tgt[:, None]).squeeze(-1)
    entr = -(lsm.exp() * lsm).sum(-1)
    go, ge = torch.randn(n, device=DEV), torch.randn(n, device=DEV)

    def run():
        if entropy:
            lp, ent = L.lm_head_logprob_entropy(h, w, tgt, rows=512)
            return (lp, ent) + torch.autograd.grad((lp, ent), (h, w), (go, ge))
        lp = L.lm_head_logprob(h, w, tgt, rows=512)
        return (lp, None) + torch.autograd.grad(lp, (h, w), go)

    lp, ent, gh, gw = run()
    if entropy:
        gr = torch.autograd.grad((lpr, entr), (hr, wr), (go, ge))
        torch.testing.assert_close(ent, entr, atol=3e-3, rtol=3e-3)
    else:
        gr = torch.autograd.grad(lpr, (hr, wr), go)
    torch.testing.assert_close(lp, lpr, atol=3e-3, rtol=3e-3)
    assert _rel(gh, gr[0]) < 2e-2
    assert _rel(gw, gr[1]) < 2e-2
    # the unfused (cuBLAS logits + row kernel) path agrees
    L.FUSED_TC = False
    try:
        lp2, ent2, gh2, gw2 = run()
    finally:
        L.FUSED_TC = True
    torch.testing.assert_close(lp, lp2, atol=2e-3, rtol=2e-3)
    assert _rel(gh, gh2) < 1e-2 and _rel(gw, gw2) < 1e-2


def test_fold_kernels():
    from thundersync_b200.ops.fold import axpby_, fold_, reduce_adjoints

    torch.manual_seed(5)
    n = 1_000_003
    g1, g2 = torch.randn(n, device=DEV), torch.randn(n, device=DEV)
    src = torch.randn(n, device=DEV)
    e1, e2 = g1.clone() + 0.7 * src, g2.clone() + src
    fold_(g1, g2, src, 0.7)
    torch.testing.assert_close(g1, e1)
    torch.testing.assert_close(g2, e2)
    out = torch.randn(n, device=DEV)
    exp = out + 0.3 * g1 - 0.2 * g2
    axpby_(out, g1, g2, 0.3, -0.2)
    torch.testing.assert_close(out, exp, atol=1e-5, rtol=1e-5)
    parts = [torch.randn(n, device=DEV) for _ in range(20)]
    base = torch.randn(n, device=DEV)
    exp = base.clone()
    for p in parts:
        exp += p
    got = reduce_adjoints(base.clone(), parts)
    torch.testing.assert_close(got, exp, atol=1e-5, rtol=1e-5)


def test_embedding_backward_deterministic():
    from thundersync_b200.ops.embedding import embedding

    torch.manual_seed(6)
    w = torch.randn(1000, 512, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    ids = torch.randint(0, 50, (4000,), device=DEV)
    y = embedding(ids, w)
    dy = torch.randn_like(y)
    (g1,) = torch.autograd.grad(y, w, dy)
    (g2,) = torch.autograd.grad(embedding(ids, w), w, dy)
    assert torch.equal(g1, g2)
    ref = torch.zeros(1000, 512, device=DEV).index_add_(0, ids, dy.float())
    assert _rel(g1, ref) < 1e-2


def test_flat_adamw_matches_torch():
    from thundersync_b200.ops.sink import ParamArena
    from thundersync_b200.parallel.optimizer import FlatAdamW

    torch.manual_seed(7)
    ps = [torch.nn.Parameter(torch.randn(37, 13, device=DEV)), torch.nn.Parameter(torch.randn(100, device=DEV))]
    ref = [torch.nn.Parameter(p.detach().clone()) for p in ps]
    arena = ParamArena(ps)
    opt = FlatAdamW(arena, lr=1e-2, weight_decay=0.1, maximize=True)
    topt = torch.optim.AdamW(ref, lr=1e-2, weight_decay=0.1, maximize=True)
    for _ in range(3):
        grads = [torch.randn_like(p) for p in ps]
        flat = arena.new_buffer()
        for p, g in zip(ps, grads):
            arena.view(flat, p).copy_(g)
        opt.step(flat)
        for p, g in zip(ref, grads):
            p.grad = g
        topt.step()
    for p, r in zip(ps, ref):
        torch.testing.assert_close(p.detach(), r.detach(), atol=1e-5, rtol=1e-5)


def test_tcgen05_descriptor_selftest():
    """One 128x128x128 UMMA tile with K-major and MN-major B operands."""
    from thundersync_b200.ops._ext import native

    torch.manual_seed(8)
    a = torch.randn(128, 128, device=DEV, dtype=torch.bfloat16)
    bk = torch.randn(128, 128, device=DEV, dtype=torch.bfloat16)
    bm = torch.randn(128, 128, device=DEV, dtype=torch.bfloat16)
    d1, d2 = native().tc_selftest(a, bk, bm)
    torch.cuda.synchronize()
    assert int(native().tc_status(a).item()) == 0
    torch.testing.assert_close(d1, a.float() @ bk.float().t(), atol=1e-2, rtol=1e-3)
    torch.testing.assert_close(d2, a.float() @ bm.float(), atol=1e-2, rtol=1e-3)


@pytest.mark.parametrize("t,s,hq,hkv,d", ATTN_CASES + [(2048, 2560, 16, 8, 128), (300, 4396, 16, 8, 128)])
def test_attention_tcgen05_forward(t, s, hq, hkv, d):
    from thundersync_b200.ops._ext import native
    from thundersync_b200.ops.attention import attention_reference

    torch.manual_seed(9)
    q = torch.randn(t, hq, d, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16)
    o, lse = native().attn_fwd_tc(q, k, v, 1 / math.sqrt(d))
    torch.cuda.synchronize()
    assert int(native().tc_status(q).item()) == 0
    orf, lser = attention_reference(q.float(), k.float(), v.float(), 1 / math.sqrt(d))
    torch.testing.assert_close(o.float(), orf, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, lser, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("d", [128, 256])
def test_attention_tcgen05_forward_growing_max(d):
    """Scores that grow along the keys: the forward's exponent reference moves only when a row's running max
    grows by more than 8 (log2 units), so P reaches up to 2^8 between moves and O is rescaled only then.
    Slopes below and above that step per key tile exercise both branches against the fp32 reference."""
    from thundersync_b200.ops._ext import native
    from thundersync_b200.ops.attention import attention_reference

    torch.manual_seed(12)
    t, s, hq, hkv = 200, 1000, 4, 2
    q = torch.zeros(t, hq, d, device=DEV)
    q[:, :, 0] = 1.0
    k = torch.randn(s, hkv, d, device=DEV) * 0.1
    # score of key j ~ slope * j (per head): gentle growth for one KV head, steep for the other
    slope = torch.tensor([0.02, 0.3], device=DEV)
    k[:, :, 0] = torch.arange(s, device=DEV)[:, None] * slope[None, :] * math.sqrt(d)
    q, k = q.to(torch.bfloat16), k.to(torch.bfloat16)
    v = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16)
    o, lse = native().attn_fwd_tc(q, k, v, 1 / math.sqrt(d))
    torch.cuda.synchronize()
    assert int(native().tc_status(q).item()) == 0
    orf, lser = attention_reference(q.float(), k.float(), v.float(), 1 / math.sqrt(d))
    torch.testing.assert_close(o.float(), orf, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, lser, atol=2e-3, rtol=1e-3)


@pytest.mark.parametrize("t,s,hq,hkv,d", ATTN_CASES + [(2048, 2560, 16, 8, 128), (300, 4396, 16, 8, 128)])
def test_attention_tcgen05_backward(t, s, hq, hkv, d):
    from thundersync_b200.ops._ext import native
    from thundersync_b200.ops.attention import attention_reference

    torch.manual_seed(10)
    q = torch.randn(t, hq, d, device=DEV, dtype=torch.bfloat16)
    k = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16)
    v = torch.randn(s, hkv, d, device=DEV, dtype=torch.bfloat16)
    scale = 1 / math.sqrt(d)
    o, lse = native().attn_fwd_tc(q, k, v, scale)
    do = torch.randn_like(o)
    dq, dk, dv = native().attn_bwd_tc(do, q, k, v, o, lse, scale)
    torch.cuda.synchronize()
    assert int(native().tc_status(q).item()) == 0
    qr, kr, vr = (x.float().requires_grad_(True) for x in (q, k, v))
    orf, _ = attention_reference(qr, kr, vr, scale)
    gq, gk, gv = torch.autograd.grad(orf, (qr, kr, vr), do.float())
    assert _rel(dq, gq) < 2e-2
    assert _rel(dk, gk) < 2e-2
    assert _rel(dv, gv) < 2e-2
    dq2, dk2, dv2 = native().attn_bwd_tc(do, q, k, v, o, lse, scale)
    assert torch.equal(dq, dq2) and torch.equal(dk, dk2) and torch.equal(dv, dv2)


@pytest.mark.parametrize("kernel", ["pair", "pair_tma_store", "wide", "single"])
@pytest.mark.parametrize("m,n,k", [(256, 512, 128), (304, 200, 72), (2304, 4096, 2048), (128, 151936 // 8, 256),
                                   (600, 1288, 264)])
@pytest.mark.parametrize("a_t,b_t", [(False, True), (False, False), (True, False), (True, True)])
def test_gemm_tcgen05(m, n, k, a_t, b_t, kernel):
    """Single-CTA, CTA-pair (cta_group::2, 256 x 256 tiles; register or TMA-store epilogue) and wide CTA-pair
    (256 x 512 tiles) kernels against an fp32 PyTorch matmul."""
    from thundersync_b200.ops._ext import native

    prev = native().gemm_tc_pair(0 if kernel == "single" else 1)
    prev_w = native().gemm_tc_wide(2 if kernel == "wide" else 0)
    prev_d = native().gemm_tc_direct(0 if kernel == "pair_tma_store" else 1)
    try:
        _check_gemm(m, n, k, a_t, b_t)
    finally:
        native().gemm_tc_pair(prev)
        native().gemm_tc_wide(prev_w)
        native().gemm_tc_direct(prev_d)


@pytest.mark.parametrize("pair", [True, False])
def test_gemm_tcgen05_two_sources(pair):
    """out = a·b + a2·b2 in one main loop (second K range from a second operand pair)."""
    from thundersync_b200.ops._ext import native

    prev = native().gemm_tc_pair(1 if pair else 0)
    try:
        torch.manual_seed(5)
        for m, n, k, k2, b_t in ((300, 384, 512, 16, True), (2304, 4096, 4096, 64, True), (1000, 512, 256, 64, False)):
            a = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
            a2 = torch.randn(m, k2, device=DEV, dtype=torch.bfloat16)
            b = torch.randn((n, k) if b_t else (k, n), device=DEV, dtype=torch.bfloat16)
            b2 = torch.randn((n, k2) if b_t else (k2, n), device=DEV, dtype=torch.bfloat16)
            bf = b.float().t() if b_t else b.float()
            b2f = b2.float().t() if b_t else b2.float()
            ref = a.float() @ bf + a2.float() @ b2f
            out = torch.empty(m, n, device=DEV)
            native().gemm_tc_cat(out, a, b, a2, b2, False, b_t, 1, 1.0)
            assert _rel(out, ref) < 1e-5, (m, n, k, k2, b_t)
    finally:
        native().gemm_tc_pair(prev)


def _check_gemm(m, n, k, a_t, b_t):
    from thundersync_b200.ops.gemm import gemm, gemm_accumulate

    torch.manual_seed(m + n + k)
    a = torch.randn((k, m) if a_t else (m, k), device=DEV, dtype=torch.bfloat16)
    b = torch.randn((n, k) if b_t else (k, n), device=DEV, dtype=torch.bfloat16)
    ref = (a.float().t() if a_t else a.float()) @ (b.float().t() if b_t else b.float())
    got = gemm(a, b, a_t=a_t, b_t=b_t, out_dtype=torch.float32)
    assert _rel(got, ref) < 1e-5
    got16 = gemm(a, b, a_t=a_t, b_t=b_t, alpha=0.5)
    assert _rel(got16, 0.5 * ref) < 1e-2
    acc = torch.ones(m, n, device=DEV)
    gemm_accumulate(acc, a, b, a_t=a_t, b_t=b_t, alpha=2.0)
    assert _rel(acc, 1.0 + 2.0 * ref) < 1e-5
    # residual operand added in the epilogue (out = a·b + R, one rounding)
    res = torch.randn(m, n, device=DEV, dtype=torch.bfloat16)
    got_r = gemm(a, b, a_t=a_t, b_t=b_t, residual=res)
    assert _rel(got_r, ref + res.float()) < 1e-2
    # output rows inside a wider buffer (row stride > N): the TMA store writes only the view
    wide = torch.full((m, n + 8), 3.0, device=DEV)
    gemm(a, b, a_t=a_t, b_t=b_t, out_dtype=torch.float32, out=wide[:, :n])
    assert _rel(wide[:, :n], ref) < 1e-5 and bool((wide[:, n:] == 3.0).all())
    from thundersync_b200.ops._ext import native

    assert int(native().tc_status(a).item()) == 0


@pytest.mark.parametrize("fused", [True, False])
def test_lora_linear_cuda_bf16_matches_fp32(fused):
    """The CUDA bf16 LoRA path (one two-source tcgen05 GEMM, or library GEMMs) against fp32 math."""
    from thundersync_b200.ops import lora as L
    from thundersync_b200.ops.lora import _LoRALinear

    L.FUSED_TC = fused
    try:
        _check_lora()
    finally:
        L.FUSED_TC = True


def _check_lora():
    from thundersync_b200.ops.lora import _LoRALinear

    torch.manual_seed(21)
    t, din, dout, r, s = 300, 512, 384, 16, 2.0
    x = torch.randn(t, din, device=DEV, dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(dout, din, device=DEV) / din ** 0.5).to(torch.bfloat16)
    a = (torch.randn(r, din, device=DEV) / din ** 0.5).requires_grad_(True)
    b = (torch.randn(dout, r, device=DEV) / r ** 0.5).requires_grad_(True)
    y = _LoRALinear.apply(x, w, a, b, s)
    dy = torch.randn_like(y)
    gx, ga, gb = torch.autograd.grad(y, (x, a, b), dy)
    xr = x.detach().float().requires_grad_(True)
    ar, br = a.detach().clone().requires_grad_(True), b.detach().clone().requires_grad_(True)
    yr = xr @ w.float().t() + s * (xr @ ar.t()) @ br.t()
    gxr, gar, gbr = torch.autograd.grad(yr, (xr, ar, br), dy.float())
    assert _rel(y, yr) < 1e-2
    assert _rel(gx, gxr) < 1e-2 and _rel(ga, gar) < 1e-2 and _rel(gb, gbr) < 1e-2
    assert ga.dtype == torch.float32 and gb.dtype == torch.float32


@pytest.mark.parametrize("n_adj,dtype", [(3, torch.float32), (16, torch.float32), (37, torch.float32),
                                         (5, torch.bfloat16)])
def test_boundary_adjoint_native_fixed_order(n_adj, dtype):
    """The native boundary-adjoint reduction adds in a fixed order into fp32 and rounds once: it equals a host
    fp32 accumulation in the same order bitwise, and repeated runs agree bitwise."""
    from thundersync_b200.engine.boundary_adjoint import reduce_boundary_adjoints

    torch.manual_seed(n_adj)
    shape = (257, 129)
    adj = [torch.randn(shape, device=DEV).to(dtype) for _ in range(n_adj)]
    existing = torch.randn(shape, device=DEV).to(dtype)
    got = reduce_boundary_adjoints(adj, existing=existing, backend="native")
    acc = existing.float().cpu().clone()
    for a in adj:
        acc += a.float().cpu()
    assert got.dtype == dtype
    assert torch.equal(got.cpu(), acc.to(dtype))
    again = reduce_boundary_adjoints(adj, existing=existing, backend="native")
    assert torch.equal(got, again)
    assert torch.equal(reduce_boundary_adjoints([None, adj[0]], backend="native").cpu(), adj[0].cpu())


def test_index_checks_record_out_of_range_ids_without_faulting():
    """Token and target ids outside their tables are skipped on the device and reported to the host."""
    from thundersync_b200.ops._ext import native

    ext = native()
    ext.bounds_status(True)  # clear anything an earlier test left
    vocab, d = 64, 128
    target = torch.zeros(vocab, d, device=DEV)
    ids = torch.tensor([3, 70, 3, 5], device=DEV, dtype=torch.long)  # 70 is outside the 64-row table
    dy = torch.ones(4, d, device=DEV, dtype=torch.bfloat16)
    ext.embedding_bwd_accumulate(target, ids, dy, 1.0)
    torch.cuda.synchronize()
    status = ext.bounds_status(True)
    assert status == {"rowops": (1, 70)}, status
    assert torch.equal(target[3], torch.full((d,), 2.0, device=DEV)) and torch.equal(target[5], torch.ones(d, device=DEV))
    logits = torch.randn(3, 256, device=DEV)
    tgt = torch.tensor([1, -2, 255], device=DEV, dtype=torch.long)
    lp, lse, _ = ext.lse_gather(logits, tgt, False)
    torch.cuda.synchronize()
    assert ext.bounds_status(True) == {"fold": (2, -2)}
    ref = torch.log_softmax(logits, -1)
    assert torch.isnan(lp[1]) and torch.allclose(lp[0], ref[0, 1], atol=1e-5) and torch.allclose(lp[2], ref[2, 255], atol=1e-5)
    assert ext.bounds_status(False) == {}
