"""The chunked (WY-form) gated delta rule and its hand-derived backward against
autograd through the token recurrence (fp64, CPU)."""

from __future__ import annotations

import pytest
import torch

from thundersync_b200.ops.gdn_chunked import chunked_backward, chunked_forward


def _recurrence64(q, k, v, g, beta, s):
    """The token recurrence in the inputs' dtype (fp64 here), as the fp32 reference computes it."""
    t, h, dk = q.shape
    qf = q * torch.rsqrt((q * q).sum(-1, keepdim=True) + 1e-6) * dk ** -0.5
    kf = k * torch.rsqrt((k * k).sum(-1, keepdim=True) + 1e-6)
    outs = []
    for i in range(t):
        s = s * g[i].exp()[:, None, None]
        kv = torch.einsum("hk,hkv->hv", kf[i], s)
        delta = (v[i] - kv) * beta[i][:, None]
        s = s + kf[i][:, :, None] * delta[:, None, :]
        outs.append(torch.einsum("hk,hkv->hv", qf[i], s))
    return torch.stack(outs, 0), s


@pytest.mark.parametrize("t,chunk", [(37, 16), (64, 16), (5, 16), (70, 64)])
def test_chunked_gdn_matches_recurrence(t, chunk):
    torch.manual_seed(t + chunk)
    h, dk, dv = 2, 16, 12
    dt = torch.float64
    q = torch.randn(t, h, dk, dtype=dt)
    k = torch.randn(t, h, dk, dtype=dt)
    v = torch.randn(t, h, dv, dtype=dt)
    g = -torch.rand(t, h, dtype=dt) * 0.5
    beta = torch.rand(t, h, dtype=dt)
    s0 = torch.randn(h, dk, dv, dtype=dt) * 0.3
    ins = [x.clone().requires_grad_(True) for x in (q, k, v, g, beta, s0)]
    o_ref, fin_ref = _recurrence64(*ins)
    do = torch.randn_like(o_ref)
    dfin = torch.randn_like(fin_ref)
    grads = torch.autograd.grad((o_ref, fin_ref), ins, (do, dfin))
    o, fin, saved = chunked_forward(q, k, v, g, beta, s0, chunk=chunk)
    assert torch.allclose(o, o_ref, atol=1e-10, rtol=1e-9)
    assert torch.allclose(fin, fin_ref.to(dt), atol=1e-10, rtol=1e-9)
    mine = chunked_backward(q, k, v, g, beta, saved, do, dfin, chunk=chunk)
    for name, a, b in zip(("dq", "dk", "dv", "dg", "dbeta", "dstate"), mine, grads):
        assert torch.allclose(a, b, atol=1e-9, rtol=1e-8), (name, float((a - b).abs().max()))
