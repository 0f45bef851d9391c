"""GPU numerics of the Gated DeltaNet kernels against fp32 torch references.

Reference behaviour: the causal conv1d + SiLU and recurrent gated delta rule
the reference evaluates for Qwen3.5 linear-attention layers
(src/thundersync/engine/streaming.py:1966-2026).
"""

from __future__ import annotations

import pytest
import torch

from thundersync_b200.ops.gdn import (causal_conv1d_reference, causal_conv1d_silu, gated_delta_rule,
                                      gated_delta_rule_reference)

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("t", [1, 37, 300])
def test_conv1d_silu_matches_reference(t):
    torch.manual_seed(t)
    c = 640
    x = torch.randn(t, c, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn(c, 4, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_(True)
    tail = torch.randn(3, c, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    y, nt = causal_conv1d_silu(x, w, tail)
    dy = torch.randn_like(y)
    dnt = torch.randn_like(nt)
    torch.autograd.backward((y, nt), (dy, dnt))
    xr, wr, tr = (a.detach().float().requires_grad_(True) for a in (x, w, tail))
    yr, ntr = causal_conv1d_reference(xr, wr, tr)
    torch.autograd.backward((yr, ntr), (dy.float(), dnt.float()))
    assert _rel(y, yr) < 1e-2
    assert torch.equal(nt.float(), ntr.float())
    assert _rel(x.grad, xr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-2
    assert _rel(tail.grad, tr.grad) < 1e-2


@pytest.mark.parametrize("t,h", [(5, 2), (130, 3), (257, 4)])
def test_gated_delta_rule_matches_reference(t, h):
    torch.manual_seed(7 * t + h)
    d = 128
    q = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = (-torch.rand(t, h, device="cuda") * 0.3).requires_grad_(True)
    beta = torch.rand(t, h, device="cuda").requires_grad_(True)
    s0 = (torch.randn(h, d, d, device="cuda") * 0.05).requires_grad_(True)
    o, fin = gated_delta_rule(q, k, v, g, beta, s0)
    do = torch.randn_like(o)
    dfin = torch.randn_like(fin) * 0.1
    torch.autograd.backward((o, fin), (do, dfin))
    ins = [a.detach().float().requires_grad_(True) for a in (q, k, v, g, beta, s0)]
    orf, finr = gated_delta_rule_reference(*ins)
    orf = orf.float()
    torch.autograd.backward((orf, finr), (do.float(), dfin))
    assert _rel(o, orf) < 1e-2
    assert _rel(fin, finr) < 1e-3
    for got, ref in zip((q, k, v, g, beta, s0), ins):
        assert _rel(got.grad, ref.grad) < 2e-2, (got.shape, _rel(got.grad, ref.grad))


@pytest.mark.parametrize("t,h", [(1000, 3), (64, 2), (129, 1)])
def test_chunked_gated_delta_rule_matches_recurrent_kernels(t, h):
    """The chunked WY-form kernels against the token-recurrent kernels and the fp32 reference."""
    from thundersync_b200.ops import gdn as G

    torch.manual_seed(11 * t + h)
    d = 128
    q = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    k = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    v = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    g = (-torch.rand(t, h, device="cuda") * 0.2).requires_grad_(True)
    beta = torch.rand(t, h, device="cuda").requires_grad_(True)
    s0 = (torch.randn(h, d, d, device="cuda") * 0.05).requires_grad_(True)
    do = torch.randn(t, h, d, device="cuda", dtype=torch.bfloat16)
    dfin = torch.randn(h, d, d, device="cuda") * 0.1
    res = []
    for chunked in (True, False):
        G.CHUNKED = chunked
        try:
            o, fin = G.gated_delta_rule(q, k, v, g, beta, s0)
            grads = torch.autograd.grad((o, fin), (q, k, v, g, beta, s0), (do, dfin))
        finally:
            G.CHUNKED = True
        res.append((o, fin) + tuple(grads))
    ins = [a.detach().float().requires_grad_(True) for a in (q, k, v, g, beta, s0)]
    orf, finr = gated_delta_rule_reference(*ins)
    gr = torch.autograd.grad((orf.float(), finr), ins, (do.float(), dfin))
    assert _rel(res[0][0], orf) < 1e-2
    assert _rel(res[0][1], finr) < 1e-3
    for a, b, r in zip(res[0][2:], res[1][2:], gr):
        assert _rel(a, r) < 2e-2, (a.shape, _rel(a, r), _rel(b, r))
