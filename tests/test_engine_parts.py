"""Boundary-adjoint reduction, canonical gradient reduction, ZeRO-1 sharded step.

Reference behaviour: tests/test_boundary_adjoint.py, tests/test_objective_ready*.py
and tests/test_sharded_step.py of the reference (CPU, fake collectives).
"""

from __future__ import annotations

import itertools
import random
import threading

import pytest
import torch

from thundersync_b200.engine.boundary_adjoint import reduce_boundary_adjoints
from thundersync_b200.engine.objective_ready import CanonicalGradientReducer, canonical_source_key
from thundersync_b200.engine.sharded_step import Collectives, ShardedOptimizerStep, partition_contiguous_by_numel


def test_reduce_boundary_adjoints_semantics():
    a, b = torch.randn(3, 4), torch.randn(3, 4)
    e = torch.randn(3, 4)
    assert reduce_boundary_adjoints([None, None]) is None
    out = reduce_boundary_adjoints([a, None, b], existing=e)
    assert torch.equal(out, (e.clone().add_(a)).add_(b))
    assert torch.equal(reduce_boundary_adjoints([a], backend="native"), a)
    with pytest.raises(ValueError):
        reduce_boundary_adjoints([a, torch.randn(2)])
    with pytest.raises(ValueError):
        reduce_boundary_adjoints([a], backend="bogus")
    x = a.clone().requires_grad_(True)
    y = reduce_boundary_adjoints([x, b], existing=e)
    (g,) = torch.autograd.grad(y.sum(), x)
    assert torch.equal(g, torch.ones_like(a))


def test_canonical_key_total_order_and_errors():
    keys = [("g", 1), 3, "a", (2, "t"), 1]
    assert sorted(keys, key=canonical_source_key) == [1, 3, "a", (2, "t"), ("g", 1)]
    with pytest.raises(TypeError):
        canonical_source_key(True)
    with pytest.raises(TypeError):
        canonical_source_key(1.5)


def test_canonical_reducer_is_arrival_order_independent():
    torch.manual_seed(0)
    sources = [(g, t) for g in range(3) for t in range(4)]
    contribs = {s: [torch.randn(5, 7) * 10 ** random.Random(hash(s)).randint(-3, 3), torch.randn(11)] for s in sources}
    results = []
    for seed in range(4):
        order = sources[:]
        random.Random(seed).shuffle(order)
        red = CanonicalGradientReducer(2)
        for s in order:
            red.add(s, contribs[s])
        results.append(red.finalize())
        assert red.diagnostics()["finalized"]
    for r in results[1:]:
        for x, y in zip(results[0], r):
            assert torch.equal(x, y)
    with pytest.raises(RuntimeError):
        red.add((0, 0), contribs[(0, 0)])


def _brute_partition(numels, w):
    total = sum(numels)
    best, best_err = None, None
    # the rule: each cut nearest its ideal point, earliest on ties, sequentially constrained
    cuts = [0]
    pre = list(itertools.accumulate(numels))
    for s in range(1, w):
        target = total * s / w
        lo, hi = cuts[-1] + 1, len(numels) - (w - s)
        c = min(range(lo, hi + 1), key=lambda c: (abs(pre[c - 1] - target), c))
        cuts.append(c)
    cuts.append(len(numels))
    return tuple(zip(cuts[:-1], cuts[1:]))


def test_partition_matches_rule():
    rng = random.Random(1)
    for _ in range(300):
        n = rng.randint(1, 12)
        w = rng.randint(1, n)
        numels = [rng.randint(1, 50) for _ in range(n)]
        assert partition_contiguous_by_numel(numels, w) == _brute_partition(numels, w)
    with pytest.raises(ValueError):
        partition_contiguous_by_numel([1], 2)


class _ThreadCollectives(Collectives):
    """W ranks as threads over shared slots; each call is a rendezvous."""

    def __init__(self, world: int) -> None:
        self.world = world
        self.barrier = threading.Barrier(world)
        self.slots: list = [None] * world

    def view(self, rank: int):
        outer = self

        class _V(Collectives):
            def _exchange(self, value):
                outer.barrier.wait()
                outer.slots[rank] = value
                outer.barrier.wait()
                got = list(outer.slots)
                outer.barrier.wait()
                return got

            def all_reduce_average_(self, t):
                got = self._exchange(t.clone())
                t.copy_(sum(got) / outer.world)

            def broadcast_(self, t, src):
                got = self._exchange(t.clone())
                t.copy_(got[src])

            def all_gather_(self, outs, t):
                got = self._exchange(t.clone())
                for o, g in zip(outs, got):
                    o.copy_(g)

        return _V()


def test_sharded_step_equals_unsharded_adamw():
    torch.manual_seed(0)
    shapes = [(4, 3), (7,), (2, 2), (5, 5), (3,)]
    base = [torch.randn(s) for s in shapes]
    grads = [[torch.randn(s) for s in shapes] for _ in range(2)]  # per-rank grads
    # unsharded reference: average grads, clip, AdamW
    ref = [torch.nn.Parameter(b.clone()) for b in base]
    for p, g0, g1 in zip(ref, grads[0], grads[1]):
        p.grad = (g0 + g1) / 2
    torch.nn.utils.clip_grad_norm_(ref, 0.5, foreach=False)
    torch.optim.AdamW(ref, lr=0.1, foreach=False).step()
    coll = _ThreadCollectives(2)
    outs, errs = {}, []

    def rank_fn(r):
        try:
            params = [torch.nn.Parameter(b.clone()) for b in base]
            step = ShardedOptimizerStep([(f"p{i}", p) for i, p in enumerate(params)],
                                        lambda ps: torch.optim.AdamW(ps, lr=0.1, foreach=False),
                                        world_size=2, rank=r, collectives=coll.view(r), grad_clip=0.5)
            for p, g in zip(params, grads[r]):
                p.grad = g.clone()
            stats = step.step()
            outs[r] = ([p.detach().clone() for p in params], stats)
        except Exception as exc:  # pragma: no cover - surfaced below
            errs.append(exc)
            coll.barrier.abort()

    ts = [threading.Thread(target=rank_fn, args=(r,)) for r in range(2)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert not errs, errs
    for r in range(2):
        for got, want in zip(outs[r][0], ref):
            assert torch.allclose(got, want.detach(), atol=1e-6)
    assert outs[0][1]["owned_param_count"] + outs[1][1]["owned_param_count"] == len(shapes)


def test_single_node_dense_layer_matches_op_by_op():
    """The one-node layer op gives bitwise the op-by-op values and gradients (CPU)."""
    from tests.grpo_fixtures import build_model
    from thundersync_b200.engine.layers import Executor, Segment

    model = build_model(0)
    ids = torch.randint(0, 512, (20,))
    pos = torch.arange(20)
    res = []
    for fused in (True, False):
        model.zero_grad(set_to_none=True)
        ex = Executor(model)
        ex.fused_layers = fused
        # two segments: a 8-token prompt whose K/V the 12-token continuation reads
        h0, st0 = ex.run(ids[:8], pos[:8], [Segment(0, 8, [])])
        past = st0[0]
        h1, _ = ex.run(ids[8:], pos[8:], [Segment(0, 12, [([k], [v]) for (k, v) in past])])
        (h0.square().sum() + h1.pow(3).sum()).backward()
        res.append((h1.detach(), {n: p.grad.clone() for n, p in model.named_parameters()}))
    assert torch.equal(res[0][0], res[1][0])
    for n in res[0][1]:
        assert torch.equal(res[0][1][n], res[1][1][n]), n
