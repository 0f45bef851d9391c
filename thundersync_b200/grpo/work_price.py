"""Trajectory work prices and longest-processing-time placement (C42).

A price is a trajectory's training work in token units: one per turn token
(linear layers) plus ``attention_weight`` per attended token pair, where the
weight is layers x heads x head_dim / parameters. ``lpt_assign`` places items
in decreasing price on the least-loaded rank (ties by item id, then rank), so
every rank that reads the same prices computes the same placement. Same
formulas as reference src/thundersync/grpo/work_price.py:20-66.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from typing import Any

__all__ = ["attention_weight", "lpt_assign", "trajectory_price"]


def trajectory_price(prompt_tokens: int, turn_tokens: int, attention_weight: float) -> int:
    if prompt_tokens < 0 or turn_tokens < 0 or attention_weight < 0:
        raise ValueError("a price takes non-negative sizes")
    total = prompt_tokens + turn_tokens
    pairs = total * total - prompt_tokens * prompt_tokens
    return int(math.ceil(turn_tokens + attention_weight * pairs))


def attention_weight(config: Any, parameter_count: int) -> float:
    if parameter_count < 1:
        raise ValueError("the model has no parameters")
    heads = int(config.num_attention_heads)
    head_dim = int(getattr(config, "head_dim", None) or config.hidden_size // heads)
    return int(config.num_hidden_layers) * heads * head_dim / float(parameter_count)


def lpt_assign(prices: Sequence[tuple[int, int]], ranks: int) -> dict[int, int]:
    if ranks < 1:
        raise ValueError("placement needs at least one rank")
    ids = [int(i) for i, _ in prices]
    if len(ids) != len(set(ids)):
        raise ValueError("an item appears twice in the placement")
    for _, p in prices:
        if p < 0:
            raise ValueError("a price must not be negative")
    loads = [0] * ranks
    out: dict[int, int] = {}
    for item, price in sorted(prices, key=lambda x: (-int(x[1]), int(x[0]))):
        r = min(range(ranks), key=lambda i: (loads[i], i))
        out[int(item)] = r
        loads[r] += int(price)
    return out
