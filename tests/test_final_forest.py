"""Final-forest micro-batches: exactness, the out-of-memory ladder and transactional deposits.

Reference behaviour: src/thundersync/grpo/final_forest.py:182-434 (halving on OOM, resume without double
counting, bounded attention cache). Out-of-memory errors are injected on the host (a micro-batch raises
torch.OutOfMemoryError after its backward already deposited part of its gradient); no device memory is
ever exhausted.
"""

from __future__ import annotations

import random

import pytest
import torch

import thundersync_b200.grpo.final_forest as ff
from tests.grpo_fixtures import build_model
from thundersync_b200.engine.streaming import arena_for
from thundersync_b200.grpo.final_forest import FinalForestReport, FinalItem, backward_final_forest
from thundersync_b200.ops.sink import GradSink


def _items(seed=0, groups=2, per_group=3):
    rng = random.Random(seed)
    out = []
    tid = 0
    for g in range(groups):
        prompt = tuple(rng.randrange(512) for _ in range(8))
        for _ in range(per_group):
            turns = []
            for _ in range(rng.randint(1, 2)):
                a = [rng.randrange(512) for _ in range(rng.randint(2, 5))]
                o = [rng.randrange(512) for _ in range(rng.randint(1, 3))]
                turns.append((tuple(a + o), tuple([True] * len(a) + [False] * len(o))))
            out.append(FinalItem(g, tid, rng.uniform(-1, 1), prompt, tuple(turns)))
            tid += 1
    return out


def _sink_grad(model, items, **kw):
    arena = arena_for(model)
    buf = arena.new_buffer(torch.float32)
    sink = GradSink(arena, buf)
    rep = FinalForestReport()
    backward_final_forest(model, items, max_tokens_per_microbatch=10_000, sink=sink, report=rep, **kw)
    return buf, rep


def test_microbatching_does_not_change_the_gradient():
    model = build_model(31)
    items = _items(1)
    whole, _ = _sink_grad(model, items)
    arena = arena_for(model)
    buf = arena.new_buffer(torch.float32)
    backward_final_forest(model, items, max_tokens_per_microbatch=20, sink=GradSink(arena, buf))
    torch.testing.assert_close(buf, whole, rtol=1e-5, atol=1e-6)


def test_out_of_memory_part_way_neither_loses_nor_double_counts(monkeypatch):
    model = build_model(32)
    items = _items(2)
    ref, _ = _sink_grad(model, items)
    real = ff._microbatch
    state = {"fail": 3}

    def flaky(model_, mb, sink, **kw):
        real(model_, mb, sink, **kw)  # the backward ran and deposited ...
        if state["fail"] > 0:
            state["fail"] -= 1
            raise torch.OutOfMemoryError("injected after the deposits")  # ... then the micro-batch "failed"

    monkeypatch.setattr(ff, "_microbatch", flaky)
    got, rep = _sink_grad(model, items)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-6)
    assert rep.out_of_memory == 3 and rep.halvings >= 1 and rep.transactional


def test_single_trajectory_falls_back_to_checkpointing_with_the_attention_cache(monkeypatch):
    model = build_model(33)
    items = _items(3, groups=1, per_group=1)
    ref, _ = _sink_grad(model, items)
    real = ff._microbatch

    def no_plain(model_, mb, sink, *, checkpoint=False, cache=None, rows=None):
        if not checkpoint:
            raise torch.OutOfMemoryError("injected: the plain forest does not fit")
        real(model_, mb, sink, checkpoint=checkpoint, cache=cache, rows=rows)

    monkeypatch.setattr(ff, "_microbatch", no_plain)
    got, rep = _sink_grad(model, items)
    torch.testing.assert_close(got, ref, rtol=1e-5, atol=1e-6)
    assert rep.checkpointed == 1 and rep.attention_cache["replayed"] > 0


def test_non_transactional_sink_refuses_a_retry(monkeypatch):
    model = build_model(34)
    items = _items(4)

    def oom(*a, **k):
        raise torch.OutOfMemoryError("injected")

    monkeypatch.setattr(ff, "_microbatch", oom)
    with pytest.raises(torch.OutOfMemoryError):
        _sink_grad(model, items, transactional=False)
