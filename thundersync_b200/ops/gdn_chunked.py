"""Chunked (WY-form) gated delta rule: the algorithm the CUDA kernels implement, in plain torch.

The recurrence (per head; state ``S`` is [dk, dv]; ``q``/``k`` are L2-normalised
and ``q`` is scaled by ``dk ** -0.5``, as Qwen3.5 / FLA's
``use_qk_l2norm_in_kernel`` do; reference call site
src/thundersync/engine/streaming.py:1966-2026)::

    S_t = e^{g_t} S_{t-1} + k_t δ_tᵀ,   δ_t = β_t (v_t − e^{g_t} S_{t-1}ᵀ k_t),   o_t = S_tᵀ q_t

Over a chunk of C steps that starts from state ``S0``, with ``G`` the
inclusive cumulative sum of ``g`` inside the chunk and ``γ = G_C``::

    A_ij = β_i e^{G_i−G_j} (k_i·k_j)   (i > j),   T = (I + A)^{-1}
    W = T diag(β e^G) K,   U = T diag(β) V,   δ = U − W S0
    P_ij = e^{G_i−G_j} (q_i·k_j)        (j ≤ i)
    O = diag(e^G) Q S0 + P δ
    S_C = e^γ S0 + Kᵀ diag(e^{γ−G}) δ

so the serial dependency runs over chunks (C = 64 here), not tokens. The
backward below is the hand-derived VJP of those formulas (it is what the
CUDA backward computes); ``tests/test_gdn_chunked.py`` checks both against
autograd through the token recurrence.
"""

from __future__ import annotations

import torch

CHUNK = 64


def _l2n(x: torch.Tensor, eps: float = 1e-6):
    r = torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)
    return x * r, r


def _l2n_bwd(x: torch.Tensor, r: torch.Tensor, dy: torch.Tensor) -> torch.Tensor:
    """VJP of y = x · rsqrt(|x|² + eps) given r = rsqrt(|x|² + eps)."""
    return r * dy - (r ** 3) * x * (dy * x).sum(-1, keepdim=True)


def _chunk_consts(kh: torch.Tensor, beta: torch.Tensor, g: torch.Tensor):
    """Per chunk: G (inclusive cumsum), the strictly lower A and T = (I + A)^{-1}."""
    c = kh.shape[0]
    G = torch.cumsum(g, 0)
    diff = G[:, None] - G[None, :]
    lower = torch.tril(torch.ones(c, c, dtype=torch.bool, device=kh.device), -1)
    A = torch.where(lower, beta[:, None] * torch.exp(torch.where(lower, diff, 0.0)) * (kh @ kh.t()), 0.0)
    eye = torch.eye(c, dtype=kh.dtype, device=kh.device)
    T = torch.linalg.solve_triangular(eye + A, eye, upper=False, unitriangular=True)
    return G, A, T


def chunked_forward(q, k, v, g, beta, state, chunk: int = CHUNK):
    """[T, H, d] inputs, fp64/fp32 math; returns (o, final_state, saved) with per-chunk start states."""
    t, h, dk = q.shape
    dv = v.shape[-1]
    qn, rq = _l2n(q)
    qh = qn * dk ** -0.5
    kh, rk = _l2n(k)
    o = torch.empty(t, h, dv, dtype=q.dtype, device=q.device)
    S = state.clone()
    starts = []
    deltas = torch.empty(t, h, dv, dtype=q.dtype, device=q.device)
    for c0 in range(0, t, chunk):
        c1 = min(t, c0 + chunk)
        starts.append(S.clone())
        for hh in range(h):
            K, Q, V = kh[c0:c1, hh], qh[c0:c1, hh], v[c0:c1, hh]
            b, gg = beta[c0:c1, hh], g[c0:c1, hh]
            G, A, T = _chunk_consts(K, b, gg)
            eG = torch.exp(G)
            W = T @ ((b * eG)[:, None] * K)
            U = T @ (b[:, None] * V)
            S0 = S[hh]
            d = U - W @ S0
            cc = c1 - c0
            incl = torch.tril(torch.ones(cc, cc, dtype=torch.bool, device=q.device))
            diff = G[:, None] - G[None, :]
            P = torch.where(incl, torch.exp(torch.where(incl, diff, 0.0)) * (Q @ K.t()), 0.0)
            o[c0:c1, hh] = eG[:, None] * (Q @ S0) + P @ d
            gam = G[-1]
            S[hh] = torch.exp(gam) * S0 + K.t() @ (torch.exp(gam - G)[:, None] * d)
            deltas[c0:c1, hh] = d
    saved = (qn, rq, kh, rk, torch.stack(starts, 0), deltas)
    return o, S, saved


def chunked_backward(q, k, v, g, beta, saved, do, dfinal, chunk: int = CHUNK):
    """Hand-derived VJP of ``chunked_forward``: (dq, dk, dv, dg, dbeta, dstate)."""
    t, h, dk = q.shape
    qn, rq, kh, rk, starts, deltas = saved
    qh = qn * dk ** -0.5
    dqh = torch.zeros_like(q)
    dkh = torch.zeros_like(k)
    dv_ = torch.zeros_like(v)
    dG_all = torch.zeros_like(g)
    dbeta = torch.zeros_like(beta)
    dS = dfinal.clone()
    n_chunks = (t + chunk - 1) // chunk
    for ci in reversed(range(n_chunks)):
        c0, c1 = ci * chunk, min(t, ci * chunk + chunk)
        cc = c1 - c0
        for hh in range(h):
            K, Q, V = kh[c0:c1, hh], qh[c0:c1, hh], v[c0:c1, hh]
            b, gg = beta[c0:c1, hh], g[c0:c1, hh]
            S0 = starts[ci, hh]
            d = deltas[c0:c1, hh]
            dO = do[c0:c1, hh]
            dSp = dS[hh]
            G, A, T = _chunk_consts(K, b, gg)
            eG = torch.exp(G)
            gam = G[-1]
            eR = torch.exp(gam - G)
            incl = torch.tril(torch.ones(cc, cc, dtype=torch.bool, device=q.device))
            diff = G[:, None] - G[None, :]
            Ed = torch.exp(torch.where(incl, diff, 0.0))
            QK = Q @ K.t()
            P = torch.where(incl, Ed * QK, 0.0)
            # gradient reaching the deltas
            dd = P.t() @ dO + eR[:, None] * (K @ dSp)
            dz = T.t() @ dd                       # (I + A)ᵀ dz = dd
            dR = b[:, None] * dz
            KS = K @ S0
            R = V - eG[:, None] * KS
            dA = -(dz @ d.t())
            lower = torch.tril(torch.ones(cc, cc, dtype=torch.bool, device=q.device), -1)
            dA = torch.where(lower, dA, 0.0)
            KK = K @ K.t()
            El = torch.exp(torch.where(lower, diff, 0.0))
            AdA = dA * torch.where(lower, b[:, None] * El * KK, 0.0)   # dA ⊙ A
            dM = dA * b[:, None] * El                                  # w.r.t. k_i·k_j
            dP = torch.where(incl, dO @ d.t(), 0.0)
            PdP = dP * P
            dN = dP * Ed                                               # w.r.t. q_i·k_j
            # values, gates
            dv_[c0:c1, hh] = dR
            dbeta[c0:c1, hh] = (dz * R).sum(-1) + (dA * torch.where(lower, El * KK, 0.0)).sum(-1)
            # keys and queries
            dK = (-(eG[:, None] * dR) @ S0.t() + dM @ K + dM.t() @ K + dN.t() @ Q
                  + eR[:, None] * (d @ dSp.t()))
            dQ = eG[:, None] * (dO @ S0.t()) + dN @ K
            dqh[c0:c1, hh] = dQ
            dkh[c0:c1, hh] = dK
            # log-decay cumsum G
            QS = Q @ S0
            dG = (-(eG[:, None] * KS * dR).sum(-1) + AdA.sum(-1) - AdA.sum(0)
                  + (dO * eG[:, None] * QS).sum(-1) + PdP.sum(-1) - PdP.sum(0))
            E = eR * ((K @ dSp) * d).sum(-1)
            dgam = torch.exp(gam) * (S0 * dSp).sum() + E.sum()
            dG = dG - E
            dG[-1] = dG[-1] + dgam
            dG_all[c0:c1, hh] = torch.flip(torch.cumsum(torch.flip(dG, [0]), 0), [0])
            # state entering the chunk
            dS[hh] = (torch.exp(gam) * dSp + Q.t() @ (eG[:, None] * dO)
                      - K.t() @ ((eG * b)[:, None] * dz))
    dq = _l2n_bwd(q, rq, dqh * dk ** -0.5)
    dk_ = _l2n_bwd(k, rk, dkh)
    return dq, dk_, dv_, dG_all, dbeta, dS
