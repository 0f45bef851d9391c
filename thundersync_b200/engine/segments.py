"""Segment forests: trajectories as provenance-tagged segments, shared exactly (C05).

A trajectory alternates prompt / action / observation segments; each segment
carries its provenance and whether its tokens are scored. ``build_forest``
compresses the trajectories of each group into a radix tree keyed on
(token, scored) pairs, so two trajectories share a physical position only if
they agree on both the token and its scoring role. Concatenating a leaf's
root path reproduces its trajectory verbatim. Interface and semantics follow
reference src/thundersync/engine/segments.py:43-346.
"""

from __future__ import annotations

from collections.abc import Iterable, Sequence
from dataclasses import dataclass, field
from enum import Enum

__all__ = ["SegmentKind", "Segment", "Trajectory", "ForestNode", "SegmentForest", "build_forest", "unshared"]


class SegmentKind(str, Enum):
    PROMPT = "prompt"
    ACTION = "action"
    OBSERVATION = "observation"


@dataclass(frozen=True)
class Segment:
    tokens: tuple[int, ...]
    kind: SegmentKind
    scored: bool

    def __post_init__(self) -> None:
        if not self.tokens:
            raise ValueError("a segment must contain at least one token")

    def __len__(self) -> int:
        return len(self.tokens)

    @classmethod
    def prompt(cls, tokens: Iterable[int], *, scored: bool = False) -> "Segment":
        return cls(tuple(tokens), SegmentKind.PROMPT, scored)

    @classmethod
    def action(cls, tokens: Iterable[int], *, scored: bool = True) -> "Segment":
        return cls(tuple(tokens), SegmentKind.ACTION, scored)

    @classmethod
    def observation(cls, tokens: Iterable[int], *, scored: bool = False) -> "Segment":
        return cls(tuple(tokens), SegmentKind.OBSERVATION, scored)


@dataclass
class Trajectory:
    segments: list[Segment]
    group_id: int = 0
    traj_id: int = 0

    def __post_init__(self) -> None:
        if not self.segments:
            raise ValueError("a trajectory must contain at least one segment")

    @property
    def tokens(self) -> list[int]:
        return [t for s in self.segments for t in s.tokens]

    @property
    def scored_mask(self) -> list[bool]:
        return [s.scored for s in self.segments for _ in s.tokens]

    @property
    def n_tokens(self) -> int:
        return sum(len(s) for s in self.segments)

    @property
    def n_scored(self) -> int:
        return sum(len(s) for s in self.segments if s.scored)

    @property
    def n_turns(self) -> int:
        return sum(1 for s in self.segments if s.kind is SegmentKind.ACTION)

    def keyed(self) -> list[tuple[int, bool]]:
        """(token, scored) pairs: the unit of sharing."""
        return [(t, s.scored) for s in self.segments for t in s.tokens]


@dataclass
class ForestNode:
    tokens: list[int]
    scored: list[bool]
    parent: int | None
    depth: int
    trajectories: list[int]
    children: list[int] = field(default_factory=list)
    group_id: int = 0

    @property
    def n_tokens(self) -> int:
        return len(self.tokens)

    @property
    def multiplicity(self) -> int:
        return len(self.trajectories)

    @property
    def is_leaf(self) -> bool:
        return not self.children


@dataclass
class SegmentForest:
    nodes: list[ForestNode]
    roots: list[int]
    trajectories: list[Trajectory]
    leaf_of: dict[int, int]

    @property
    def physical_tokens(self) -> int:
        return sum(n.n_tokens for n in self.nodes)

    @property
    def logical_tokens(self) -> int:
        return sum(t.n_tokens for t in self.trajectories)

    @property
    def scored_tokens(self) -> int:
        return sum(sum(n.scored) * n.multiplicity for n in self.nodes)

    @property
    def physical_scored_tokens(self) -> int:
        return sum(sum(n.scored) for n in self.nodes)

    @property
    def padded_tokens(self) -> int:
        if not self.trajectories:
            return 0
        return len(self.trajectories) * max(t.n_tokens for t in self.trajectories)

    @property
    def compression(self) -> float:
        return self.logical_tokens / max(self.physical_tokens, 1)

    @property
    def max_depth(self) -> int:
        return max((n.depth for n in self.nodes), default=0)

    def path_to_root(self, node: int) -> list[int]:
        out: list[int] = []
        cur: int | None = node
        while cur is not None:
            out.append(cur)
            cur = self.nodes[cur].parent
        out.reverse()
        return out

    def stats(self) -> dict[str, float | int]:
        return {
            "trajectories": len(self.trajectories),
            "nodes": len(self.nodes),
            "logical_tokens": self.logical_tokens,
            "physical_tokens": self.physical_tokens,
            "padded_tokens": self.padded_tokens,
            "compression": round(self.compression, 4),
            "scored_tokens": self.scored_tokens,
            "scored_fraction": round(self.scored_tokens / max(self.logical_tokens, 1), 4),
            "max_depth": self.max_depth,
        }


def _common_prefix(seqs: Sequence[list[tuple[int, bool]]]) -> int:
    """Length of the longest prefix shared by every sequence (monotone -> bisect)."""
    if not seqs:
        return 0
    hi = min(len(s) for s in seqs)
    if len(seqs) == 1:
        return hi
    lo = 0
    first = seqs[0]
    while lo < hi:
        mid = (lo + hi + 1) // 2
        head = first[:mid]
        if all(s[:mid] == head for s in seqs[1:]):
            lo = mid
        else:
            hi = mid - 1
    return lo


def unshared(trajectories: Sequence[Trajectory]) -> list[Trajectory]:
    """The same trajectories with sharing disabled (each in its own group)."""
    return [Trajectory(list(t.segments), group_id=1_000_000 + i, traj_id=t.traj_id) for i, t in enumerate(trajectories)]


def build_forest(trajectories: Sequence[Trajectory]) -> SegmentForest:
    nodes: list[ForestNode] = []
    roots: list[int] = []
    leaf_of: dict[int, int] = {}
    groups: dict[int, list[Trajectory]] = {}
    for t in trajectories:
        groups.setdefault(t.group_id, []).append(t)
    for gid in sorted(groups):
        keyed = {t.traj_id: t.keyed() for t in groups[gid]}
        # explicit stack instead of recursion: (trajectory ids, offset, parent, depth)
        stack: list[tuple[list[int], int, int | None, int]] = [([t.traj_id for t in groups[gid]], 0, None, 0)]
        while stack:
            ids, offset, parent, depth = stack.pop()
            rests = [keyed[i][offset:] for i in ids]
            share = _common_prefix(rests)
            if share == 0 and parent is not None:
                raise AssertionError("zero-length non-root node")
            head = rests[0][:share]
            idx = len(nodes)
            nodes.append(ForestNode([k[0] for k in head], [k[1] for k in head], parent, depth, list(ids), group_id=gid))
            if parent is None:
                roots.append(idx)
            else:
                nodes[parent].children.append(idx)
            nxt = offset + share
            branches: dict[tuple[int, bool], list[int]] = {}
            for i in ids:
                if len(keyed[i]) == nxt:
                    leaf_of[i] = idx
                else:
                    branches.setdefault(keyed[i][nxt], []).append(i)
            # push in reverse so children are emitted in first-appearance order
            for key in reversed(list(branches)):
                stack.append((branches[key], nxt, idx, depth + 1))
    return SegmentForest(nodes, roots, list(trajectories), leaf_of)
