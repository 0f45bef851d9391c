"""Model-owned source attention objects with optional query chunking (C28).

The reference builds cuDNN-frontend SDPA graphs with a bottom-right diagonal,
cached by geometry, with optional query chunks that trim causally invisible
keys and key buckets for plan reuse (src/thundersync/grpo/attention.py:14-172).
Here the kernel is this package's tcgen05 bottom-right attention, which needs
no plans, workspaces or buckets. What is kept is the object interface and the
query-chunk semantics: with ``query_chunk`` each chunk of queries runs over
the keys it can see (ancestors plus its own causal prefix), which bounds the
backward's transient memory for very long sources.

``graph_attention(scale, query_chunk=...)`` returns ``f(q, k, v)`` on
[B, H, T, D] tensors; ``source_graph_attention(query_chunk, kv_bucket)``
returns ``attention(query, keys, values, scale)`` taking the streaming
layout: ``query`` [T, Hq, D] (or [1, Hq, T, D]) and per-chunk key/value lists
of [S_i, Hkv, D].
"""

from __future__ import annotations

import torch

from thundersync_b200.ops.attention import chunked_attention

__all__ = ["graph_attention", "source_graph_attention"]


def _bottom_right(q: torch.Tensor, keys: list[torch.Tensor], values: list[torch.Tensor], scale: float,
                  query_chunk: int) -> torch.Tensor:
    if not query_chunk or q.shape[0] <= query_chunk:
        return chunked_attention(q, keys, values, scale)
    k = torch.cat(keys, 0) if len(keys) > 1 else keys[0]
    v = torch.cat(values, 0) if len(values) > 1 else values[0]
    prefix = k.shape[0] - q.shape[0]
    outs = []
    for a in range(0, q.shape[0], query_chunk):
        b = min(a + query_chunk, q.shape[0])
        outs.append(chunked_attention(q[a:b], [k[: prefix + b]], [v[: prefix + b]], scale))
    return torch.cat(outs, 0)


def graph_attention(scale: float, *, query_chunk: int = 0, **_unused):
    """``f(q, k, v)`` on [B, H, T, D] tensors (keys may be longer: bottom-right alignment)."""

    def f(q, k, v):
        outs = []
        for i in range(q.shape[0]):
            o = _bottom_right(q[i].transpose(0, 1), [k[i].transpose(0, 1)], [v[i].transpose(0, 1)], scale,
                              query_chunk)
            outs.append(o.transpose(0, 1))
        return torch.stack(outs, 0)

    return f


def source_graph_attention(*, query_chunk: int, kv_bucket: int):
    """One model's source attention callable; ``kv_bucket`` is accepted and has no effect (no plans)."""
    if kv_bucket and not query_chunk:
        raise ValueError("kv_bucket requires query_chunk")
    records: list[dict] = []

    def attention(query, keys, values, scale):
        if query.dtype != torch.bfloat16 and query.is_cuda:
            raise RuntimeError("source attention requires bfloat16 inputs on CUDA")
        squeeze = query.dim() == 4
        q = query[0].transpose(0, 1) if squeeze else query
        out = _bottom_right(q, list(keys), list(values), float(scale), query_chunk)
        return out.transpose(0, 1)[None] if squeeze else out

    attention.planning_records = records
    return attention
