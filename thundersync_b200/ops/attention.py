"""Bottom-right causal attention of new queries over an ancestor chain (K04′).

``chunked_attention(q, k_chunks, v_chunks, scale)``: ``q`` is [T, Hq, d]; the
key/value chain is the concatenation of the chunks ([S_i, Hkv, d] each,
ancestors first, the queries' own keys last). Query ``t`` sees keys
``j <= S - T + t`` (bottom-right alignment): every ancestor key is visible
and the own chunk is causal. GQA maps query head ``h`` to KV head
``h // (Hq / Hkv)``. One autograd node holds per-chunk references, so
retention stays O(total tokens) rather than sum-of-prefixes (reference:
src/thundersync/engine/streaming.py:1314-1423, ``_ChunkedCausalSDPA``).

On CUDA the forward and backward are this package's kernels: the forward
writes ``O`` and the row log-sum-exp, the backward recomputes ``P`` from the
saved LSE (no ``S × T`` buffers) and produces dQ without atomics.
"""

from __future__ import annotations

import contextlib
import math
import threading
from typing import Any

import torch

from thundersync_b200.ops._ext import native


def attention_reference(q, k, v, scale):
    """fp32 oracle: [T,Hq,d] x [S,Hkv,d] -> ([T,Hq,d], lse [Hq,T])."""
    t, hq, d = q.shape
    s, hkv, _ = k.shape
    g = hq // hkv
    qf = q.float().transpose(0, 1)
    kf = k.float().repeat_interleave(g, dim=1).transpose(0, 1)
    vf = v.float().repeat_interleave(g, dim=1).transpose(0, 1)
    logits = torch.matmul(qf, kf.transpose(1, 2)) * scale
    qi = torch.arange(t, device=q.device)[:, None]
    kj = torch.arange(s, device=q.device)[None, :]
    mask = kj <= (s - t + qi)
    logits = logits.masked_fill(~mask, float("-inf"))
    lse = torch.logsumexp(logits, dim=-1)
    p = torch.exp(logits - lse[..., None])
    out = torch.matmul(p, vf).transpose(0, 1)
    return out.to(q.dtype), lse


class AttentionOutputCache:
    """Bounded store of attention outputs for checkpointed forwards (reference behaviour:
    src/thundersync/grpo/final_forest.py:182-239).

    Under per-layer activation checkpointing the backward recomputes each layer, attention included.
    Inside :meth:`layer` the first run of a layer *records*: every attention call keeps its output and
    row log-sum-exp while the charged bytes stay within ``budget_bytes`` (calls beyond it are declined
    and recomputed as usual). A later run of the same layer -- the recompute in the backward -- *replays*
    the calls in order and skips the kernel for every kept output. Results are bitwise those of a
    recompute: the same kernel produced them.
    """

    def __init__(self, budget_bytes: int) -> None:
        self.budget_bytes = int(budget_bytes)
        self.charged_bytes = 0
        self.saved = self.declined = self.replayed = 0
        self._layers: dict[Any, list] = {}
        self._active: list | None = None
        self._recording = False

    @contextlib.contextmanager
    def layer(self, key: Any):
        """Run one layer's body: records on the first entry for ``key``, replays on later entries."""
        first = key not in self._layers
        if first:
            self._layers[key] = []
        prev = (self._active, self._recording, getattr(_CACHE, "current", None))
        self._active = list(self._layers[key]) if not first else self._layers[key]
        self._recording = first
        _CACHE.current = self
        try:
            yield
        finally:
            self._active, self._recording, _CACHE.current = prev

    def _take(self, q: torch.Tensor):
        if self._active is None:
            return None, False
        if self._recording:
            return None, True
        if not self._active:
            raise RuntimeError("attention recompute issued more calls than the recorded forward")
        hit = self._active.pop(0)
        if hit is not None:
            self.replayed += 1
        return hit, False

    def _keep(self, out: torch.Tensor, lse: torch.Tensor) -> None:
        size = out.numel() * out.element_size() + lse.numel() * lse.element_size()
        if self.charged_bytes + size <= self.budget_bytes:
            self.charged_bytes += size
            self.saved += 1
            self._active.append((out.detach(), lse.detach()))
        else:
            self.declined += 1
            self._active.append(None)

    def report(self) -> dict[str, int]:
        return {"budget_bytes": self.budget_bytes, "charged_bytes": self.charged_bytes, "saved": self.saved,
                "declined": self.declined, "replayed": self.replayed}


_CACHE = threading.local()


class _ChunkedAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, scale, n, *kv):
        ks, vs = kv[:n], kv[n:]
        cache = getattr(_CACHE, "current", None)
        hit, record = cache._take(q) if cache is not None else (None, False)
        if hit is not None:
            out, lse = hit[0].detach(), hit[1].detach()  # fresh tensor objects over the kept storage
        else:
            k = ks[0] if n == 1 else torch.cat(ks, 0)
            v = vs[0] if n == 1 else torch.cat(vs, 0)
            if q.is_cuda:
                out, lse = native().attn_fwd_tc(q.contiguous(), k.contiguous(), v.contiguous(), float(scale))
            else:
                out, lse = attention_reference(q, k, v, scale)
            if record:
                cache._keep(out, lse)
        ctx.scale = scale
        ctx.n = n
        ctx.lens = [t.shape[0] for t in ks]
        ctx.save_for_backward(q, out, lse, *kv)
        return out

    @staticmethod
    def backward(ctx, do):
        q, out, lse, *kv = ctx.saved_tensors
        n = ctx.n
        ks, vs = kv[:n], kv[n:]
        k = ks[0] if n == 1 else torch.cat(ks, 0)
        v = vs[0] if n == 1 else torch.cat(vs, 0)
        if q.is_cuda:
            dq, dk, dv = native().attn_bwd_tc(
                do.contiguous(), q.contiguous(), k.contiguous(), v.contiguous(), out, lse, float(ctx.scale)
            )
        else:
            with torch.enable_grad():
                q_ = q.detach().requires_grad_(True)
                k_ = k.detach().requires_grad_(True)
                v_ = v.detach().requires_grad_(True)
                o_, _ = attention_reference(q_, k_, v_, ctx.scale)
                dq, dk, dv = torch.autograd.grad(o_, (q_, k_, v_), do)
        dks = list(torch.split(dk, ctx.lens, 0))
        dvs = list(torch.split(dv, ctx.lens, 0))
        grads = []
        for i, g in enumerate(dks + dvs):
            grads.append(g if ctx.needs_input_grad[3 + i] else None)
        return (dq if ctx.needs_input_grad[0] else None, None, None, *grads)


def chunked_attention(q, k_chunks, v_chunks, scale=None):
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[-1])
    if len(k_chunks) != len(v_chunks) or not k_chunks:
        raise ValueError("need matching, non-empty key and value chunk lists")
    return _ChunkedAttention.apply(q, float(scale), len(k_chunks), *k_chunks, *v_chunks)
