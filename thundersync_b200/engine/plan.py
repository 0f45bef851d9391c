"""Lay a segment forest out for execution (C06).

DFS pre-order gives every node a contiguous physical range with ancestors
first, so one traversal yields every index the step needs: token and position
ids, node geometry, ``subtree_end`` (key ``k`` is visible to query ``q`` iff
``k <= q < subtree_end[k]``), the scoring gather (``score_src`` = physical
row of each scored token's predecessor), the logical view
(``logical_to_slot``), and per-node ``key_ranges`` (ancestor spans, then the
node's own span, which alone is causal). Field names and meanings follow
reference src/thundersync/engine/plan.py:42-362.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from thundersync_b200.engine.segments import SegmentForest

__all__ = ["ExecutionPlan", "compile_plan", "visibility_mask"]

_FIELDS = ("token_ids", "position_ids", "node_of", "node_start", "node_end", "node_parent", "node_depth",
           "subtree_end", "score_src", "score_tgt", "score_pos", "logical_to_slot", "logical_traj")


@dataclass
class ExecutionPlan:
    token_ids: torch.Tensor
    position_ids: torch.Tensor
    node_of: torch.Tensor
    node_start: torch.Tensor
    node_end: torch.Tensor
    node_parent: torch.Tensor
    node_depth: torch.Tensor
    subtree_end: torch.Tensor
    score_src: torch.Tensor
    score_tgt: torch.Tensor
    score_pos: torch.Tensor
    logical_to_slot: torch.Tensor
    logical_traj: torch.Tensor
    key_ranges: list[list[tuple[int, int]]]
    forest: SegmentForest

    @property
    def n_physical(self) -> int:
        return int(self.token_ids.shape[0])

    @property
    def n_scored(self) -> int:
        return int(self.score_src.shape[0])

    @property
    def n_logical_scored(self) -> int:
        return int(self.logical_to_slot.shape[0])

    @property
    def n_nodes(self) -> int:
        return int(self.node_start.shape[0])

    @property
    def is_two_level(self) -> bool:
        return int(self.node_depth.max().item()) <= 1 if self.n_nodes else True

    def to(self, device, *, non_blocking: bool = False) -> "ExecutionPlan":
        dev = torch.device(device)
        if self.token_ids.device == dev:
            return self
        moved = {f: getattr(self, f).to(dev, non_blocking=non_blocking) for f in _FIELDS}
        return ExecutionPlan(**moved, key_ranges=self.key_ranges, forest=self.forest)

    def physical_path(self, traj_id: int) -> list[int]:
        out: list[int] = []
        for n in self.forest.path_to_root(self.forest.leaf_of[traj_id]):
            out.extend(range(int(self.node_start[n]), int(self.node_end[n])))
        return out

    def summary(self) -> dict:
        f = self.forest
        return {**f.stats(), "physical_scored": self.n_scored, "logical_scored": self.n_logical_scored,
                "two_level": self.is_two_level, "baseline_projected": f.padded_tokens,
                "projection_reduction": round(f.padded_tokens / max(self.n_scored, 1), 3)}


def compile_plan(forest: SegmentForest, device="cpu") -> ExecutionPlan:
    nodes = forest.nodes
    order: list[int] = []
    stack = list(reversed(forest.roots))
    while stack:
        n = stack.pop()
        order.append(n)
        stack.extend(reversed(nodes[n].children))
    start, end, pos0 = {}, {}, {}
    toks: list[int] = []
    poss: list[int] = []
    node_of: list[int] = []
    cur = 0
    for n in order:
        node = nodes[n]
        p = node.parent
        pos0[n] = 0 if p is None else pos0[p] + len(nodes[p].tokens)
        start[n] = cur
        cur += len(node.tokens)
        end[n] = cur
        toks.extend(node.tokens)
        poss.extend(range(pos0[n], pos0[n] + len(node.tokens)))
        node_of.extend([n] * len(node.tokens))
    sub_end: dict[int, int] = {}
    for n in reversed(order):
        sub_end[n] = max([end[n], *(sub_end[c] for c in nodes[n].children)])
    subtree = []
    for n in order:
        subtree.extend([sub_end[n]] * (end[n] - start[n]))
    key_ranges: list[list[tuple[int, int]]] = [[] for _ in nodes]
    for n in order:
        p = nodes[n].parent
        inherited = [] if p is None else key_ranges[p][:-1] + [(start[p], end[p])]
        key_ranges[n] = [(s, e) for s, e in inherited if e > s] + [(start[n], end[n])]
    src, tgt, spos = [], [], []
    slot_start, slot_count = {}, {}
    n_slots = 0
    for n in order:
        node = nodes[n]
        p = node.parent
        slot_start[n] = n_slots
        c = 0
        for j, (t, s) in enumerate(zip(node.tokens, node.scored)):
            if not s or (p is None and j == 0):
                continue
            phys = start[n] + j
            spos.append(phys)
            src.append(phys - 1 if j > 0 else end[p] - 1)
            tgt.append(t)
            c += 1
        slot_count[n] = c
        n_slots += c
    l2s, ltraj = [], []
    for traj in forest.trajectories:
        for n in forest.path_to_root(forest.leaf_of[traj.traj_id]):
            c = slot_count.get(n, 0)
            l2s.extend(range(slot_start[n], slot_start[n] + c))
            ltraj.extend([traj.traj_id] * c)

    def T(x):
        return torch.tensor(x, dtype=torch.long, device=device)

    n_all = range(len(nodes))
    return ExecutionPlan(
        token_ids=T(toks), position_ids=T(poss), node_of=T(node_of),
        node_start=T([start[n] for n in n_all]), node_end=T([end[n] for n in n_all]),
        node_parent=T([-1 if nodes[n].parent is None else nodes[n].parent for n in n_all]),
        node_depth=T([nodes[n].depth for n in n_all]), subtree_end=T(subtree),
        score_src=T(src), score_tgt=T(tgt), score_pos=T(spos), logical_to_slot=T(l2s), logical_traj=T(ltraj),
        key_ranges=key_ranges, forest=forest,
    )


def visibility_mask(plan: ExecutionPlan) -> torch.Tensor:
    """[P, P] bool mask implied by the plan (reference/testing only)."""
    p = plan.n_physical
    m = torch.zeros(p, p, dtype=torch.bool)
    for n in range(plan.n_nodes):
        s, e = int(plan.node_start[n]), int(plan.node_end[n])
        if s == e:
            continue
        for ks, ke in plan.key_ranges[n][:-1]:
            m[s:e, ks:ke] = True
        m[s:e, s:e] = torch.ones(e - s, e - s, dtype=torch.bool).tril()
    return m
