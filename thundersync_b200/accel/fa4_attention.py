"""This package's tcgen05 attention as a Hugging Face attention implementation.

The reference registers FlashAttention-4 under the name ``"fa4"`` so its
baselines run the same kernel as its streaming path
(src/thundersync/accel/fa4_attention.py:19-66). Here the registered function
runs this package's sm_100a attention kernels (bottom-right causal, GQA,
LSE-saving forward and atomics-free backward) on batch-1 packed inputs, so a
``transformers`` model loaded with ``attn_implementation="fa4"`` (or
``ATTENTION_NAME``) uses them. Attention masks other than plain causal are
refused rather than ignored.
"""

from __future__ import annotations

import torch

from thundersync_b200.ops.attention import chunked_attention

__all__ = ["ATTENTION_NAME", "fa4_attention_forward", "register_fa4_attention"]

ATTENTION_NAME = "fa4"


def fa4_attention_forward(module, query, key, value, attention_mask=None, scaling=None, dropout=0.0, **kwargs):
    """HF attention signature: q/k/v [B, H, T, D] → ([B, T, H, D], None)."""
    if dropout:
        raise ValueError("native attention has no dropout")
    if attention_mask is not None and attention_mask.dim() == 4 and not bool(
            (attention_mask == attention_mask.tril()).all()):
        raise ValueError("native attention supports causal masks only")
    outs = []
    for b in range(query.shape[0]):
        q = query[b].transpose(0, 1)
        k = key[b].transpose(0, 1)
        v = value[b].transpose(0, 1)
        outs.append(chunked_attention(q, [k], [v], scaling))
    return torch.stack(outs, 0), None


def register_fa4_attention() -> bool:
    """Register under ``ATTENTION_NAME`` with ``transformers``; False when it is absent."""
    try:
        from transformers import AttentionInterface
    except Exception:  # noqa: BLE001 - transformers is optional
        return False
    AttentionInterface.register(ATTENTION_NAME, fa4_attention_forward)
    return True
